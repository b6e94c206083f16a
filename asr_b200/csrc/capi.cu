// extern "C" entry points of the transducer losses (RNN-T, TDT): argument
// checks, workspace carving and the launch sequence of each op. The CTC entry
// points live in ctc.cu.
//
// Launch sequence (all on the caller's stream, no host synchronisation):
//   forward : lattice_prep -> joint forward (GEMM + fused log-softmax gather)
//             -> alpha recursion (loss, log_prob)
//   backward: lattice_prep -> beta recursion (posteriors, duration-logit grads)
//             -> zero the gradients -> joint backward (dlogits, dH, dW)
#include <algorithm>
#include <cstdlib>
#include <cstring>

#include "dp.cuh"
#include "joint.cuh"

using namespace asr;

namespace {

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

int64_t node_capacity(int B, int T, int U) { return (int64_t)B * T * U; }

bool bad_dims(int B, int T, int U, int V, int d) { return B < 0 || T < 1 || U < 1 || V < 1 || d < 1; }

// Layout of a transducer workspace.
struct TrWorkspace {
    LatticeMeta meta;
    float* cb = nullptr;    // backward: (cap,)
    float* ct = nullptr;    // backward: (cap,)
    float* gdur = nullptr;  // backward TDT: (cap, n_dur)
    double* beta = nullptr;  // backward: (B, T + 1, U), the TDT alpha array's shape
    void* joint = nullptr;  // joint-network scratch
    size_t joint_bytes = 0;
    // bf16 activations: fp32 copies for the SIMT path, fp32 gradient sums
    float* enc32 = nullptr;   // (B, T, d)
    float* dec32 = nullptr;   // (B, U, d)
    float* genc32 = nullptr;  // backward: (B, T, d)
    float* gdec32 = nullptr;  // backward: (B, U, d)
};

// Extra workspace for bf16 activations: fp32 copies when the SIMT joint reads
// them, and fp32 gradient sums (converted to bf16 at the end) in the backward.
struct ActStaging {
    bool copies, grads;
};

ActStaging act_staging(int act_dtype, bool tc, bool backward) {
    const bool bf16 = act_dtype == ASR_DTYPE_BF16;
    return {bf16 && !tc, bf16 && backward};
}

size_t joint_scratch_bytes(const JointArgs& a, int64_t cap, bool tc, bool backward) {
    if (tc) return backward ? tc_backward_scratch_bytes(a, (int)cap) : tc_forward_scratch_bytes(a, (int)cap);
    return backward ? simt_backward_scratch_bytes(a.V + a.n_dur, (int)cap) : 0;
}

// Elements of the TDT alpha array (B, T + 1, U); beta has the same layout.
size_t tdt_alpha_len(const JointArgs& a) { return (size_t)a.B * (a.T + 1) * a.U; }

size_t tr_workspace_bytes(const JointArgs& a, int64_t cap, bool tc, bool backward, int act_dtype = ASR_DTYPE_F32) {
    size_t n = lattice_meta_bytes(a.B);
    const ActStaging sg = act_staging(act_dtype, tc, backward);
    const size_t ne = sizeof(float) * (size_t)a.B * a.T * a.d, nd = sizeof(float) * (size_t)a.B * a.U * a.d;
    if (sg.copies) n += align256(ne) + align256(nd);
    if (sg.grads) n += align256(ne) + align256(nd);
    if (backward) {
        n += 2 * align256(sizeof(float) * cap);
        n += align256(sizeof(double) * tdt_alpha_len(a));
        if (a.n_dur > 0) n += align256(sizeof(float) * cap * a.n_dur);
    }
    n += align256(joint_scratch_bytes(a, cap, tc, backward));
    return n + 256;  // slack for aligning the base pointer
}

TrWorkspace carve(void* ws, const JointArgs& a, int64_t cap, bool tc, bool backward, int act_dtype = ASR_DTYPE_F32) {
    TrWorkspace w;
    char* p = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(ws) + 255) & ~uintptr_t(255));
    p = lattice_meta_carve(p, a.B, &w.meta);
    const ActStaging sg = act_staging(act_dtype, tc, backward);
    const size_t ne = sizeof(float) * (size_t)a.B * a.T * a.d, nd = sizeof(float) * (size_t)a.B * a.U * a.d;
    if (sg.copies) {
        w.enc32 = reinterpret_cast<float*>(p);
        p += align256(ne);
        w.dec32 = reinterpret_cast<float*>(p);
        p += align256(nd);
    }
    if (sg.grads) {
        w.genc32 = reinterpret_cast<float*>(p);
        p += align256(ne);
        w.gdec32 = reinterpret_cast<float*>(p);
        p += align256(nd);
    }
    if (backward) {
        w.cb = reinterpret_cast<float*>(p);
        p += align256(sizeof(float) * cap);
        w.ct = reinterpret_cast<float*>(p);
        p += align256(sizeof(float) * cap);
        w.beta = reinterpret_cast<double*>(p);
        p += align256(sizeof(double) * tdt_alpha_len(a));
        if (a.n_dur > 0) {
            w.gdur = reinterpret_cast<float*>(p);
            p += align256(sizeof(float) * cap * a.n_dur);
        }
    }
    w.joint = p;
    w.joint_bytes = joint_scratch_bytes(a, cap, tc, backward);
    return w;
}

JointArgs make_args(const float* enc, const float* dec, const float* W, const float* Wd, const int32_t* targets,
                    int B, int T, int U, int V, int n_dur, int d, int S, int blank, float sigma) {
    JointArgs a;
    std::memset(&a, 0, sizeof(a));
    a.enc = enc;
    a.dec = dec;
    a.W = W;
    a.Wd = Wd;
    a.targets = targets;
    a.B = B;
    a.T = T;
    a.U = U;
    a.V = V;
    a.n_dur = n_dur;
    a.d = d;
    a.S = S;
    a.blank = blank;
    a.sigma = sigma;
    a.vec = (d % 8 == 0 && reinterpret_cast<uintptr_t>(enc) % 16 == 0 && reinterpret_cast<uintptr_t>(dec) % 16 == 0)
                ? 1
                : 0;
    return a;
}

// Points the joint at the caller's activations: fp32 directly, bf16 either
// directly (tensor-core path) or through the fp32 copies in the workspace.
int bind_activations(JointArgs& a, const void* enc, const void* dec, int act_dtype, const TrWorkspace& w,
                     cudaStream_t st) {
    if (act_dtype == ASR_DTYPE_F32) {
        a.enc = static_cast<const float*>(enc);
        a.dec = static_cast<const float*>(dec);
        return ASR_OK;
    }
    const auto* e16 = static_cast<const __nv_bfloat16*>(enc);
    const auto* d16 = static_cast<const __nv_bfloat16*>(dec);
    if (w.enc32) {
        int rc = launch_bf16_to_f32(e16, w.enc32, (int64_t)a.B * a.T * a.d, st);
        if (rc) return rc;
        rc = launch_bf16_to_f32(d16, w.dec32, (int64_t)a.B * a.U * a.d, st);
        if (rc) return rc;
        a.enc = w.enc32;
        a.dec = w.dec32;
        a.vec = a.d % 8 == 0;
        return ASR_OK;
    }
    a.enc = nullptr;
    a.dec = nullptr;
    a.enc16 = e16;
    a.dec16 = d16;
    return ASR_OK;
}

// Joint path. tf32 = 1: bf16 tensor cores. tf32 = 0 (the reference's fp32
// semantics): the tensor cores on split operands (three bf16 products, fp32
// accurate; JointArgs::split), or the fp32 SIMT joint where the tensor-core
// kernels do not take the shape or ASR_B200_FP32_SIMT=1 asks for it. Sets
// a.split to the path's value.
bool fp32_simt_forced() {
    static const bool forced = [] {
        const char* e = std::getenv("ASR_B200_FP32_SIMT");
        return e && e[0] == '1';
    }();
    return forced;
}

bool use_tc(int tf32, JointArgs& a) {
    a.split = tf32 ? 0 : 1;
    if ((tf32 || !fp32_simt_forced()) && tc_supported(a)) return true;
    a.split = 0;
    return false;
}

bool use_tc_bwd(int tf32, JointArgs& a) {
    if (use_tc(tf32, a) && tc_backward_supported(a)) return true;
    a.split = 0;
    return false;
}

// The logit stash of a (forward, backward) pair: used when both directions run
// the tensor-core joint (the stash layout follows its geometry); empty otherwise.
LogitStash stash_view(int tf32, const JointArgs& a, const void* stash, size_t stash_bytes) {
    JointArgs c = a;
    if (!stash || !use_tc_bwd(tf32, c)) return LogitStash{nullptr, nullptr, 0};
    return tc_stash_carve(c, const_cast<void*>(stash), stash_bytes);
}

}  // namespace

extern "C" const char* asr_status_string(int status) {
    switch (status) {
        case ASR_OK: return "ok";
        case ASR_ERR_INVALID_ARGUMENT: return "invalid argument";
        case ASR_ERR_WORKSPACE: return "workspace missing or too small";
        case ASR_ERR_UNSUPPORTED: return "shape outside the supported kernel range";
        case ASR_ERR_CUDA: return "CUDA launch or runtime error";
        case ASR_ERR_SCRATCH_LIMIT: return "problem exceeds the fixed scratch of the allocation-free entry point";
        default: return "unknown status";
    }
}

extern "C" int asr_abi_version(void) { return 2; }

extern "C" int asr_joint_path(int tf32, int V, int n_dur, int d) {
    if (V < 1 || d < 1 || n_dur < 0) return 0;
    JointArgs a = make_args(nullptr, nullptr, nullptr, nullptr, nullptr, 1, 1, 1, V, n_dur, d, 0, 0, 0.f);
    return use_tc(tf32, a) ? 1 : 0;
}

// ------------------------------------------------------------------------ RNN-T

namespace {

int check_act_dtype(int act_dtype) {
    return act_dtype == ASR_DTYPE_F32 || act_dtype == ASR_DTYPE_BF16 ? ASR_OK : ASR_ERR_INVALID_ARGUMENT;
}

// bf16 gradient outputs: fp32 sums in the workspace, rounded to bf16 at the end.
int finish_act_grads(const JointArgs& a, const TrWorkspace& w, void* grad_encoder, void* grad_decoder,
                     cudaStream_t st) {
    if (!w.genc32) return ASR_OK;
    int rc = launch_f32_to_bf16(w.genc32, static_cast<__nv_bfloat16*>(grad_encoder), (int64_t)a.B * a.T * a.d, st);
    if (rc) return rc;
    return launch_f32_to_bf16(w.gdec32, static_cast<__nv_bfloat16*>(grad_decoder), (int64_t)a.B * a.U * a.d, st);
}

int zero_act_grads(const JointArgs& a, const TrWorkspace& w, void* grad_encoder, void* grad_decoder, float** ge,
                   float** gd, cudaStream_t st) {
    *ge = w.genc32 ? w.genc32 : static_cast<float*>(grad_encoder);
    *gd = w.gdec32 ? w.gdec32 : static_cast<float*>(grad_decoder);
    ASR_CUDA_TRY(cudaMemsetAsync(*ge, 0, sizeof(float) * (size_t)a.B * a.T * a.d, st));
    ASR_CUDA_TRY(cudaMemsetAsync(*gd, 0, sizeof(float) * (size_t)a.B * a.U * a.d, st));
    return ASR_OK;
}

size_t rnnt_workspace_impl(int B, int T, int U, int V, int d, int tf32, int backward, int act_dtype) {
    if (bad_dims(B, T, U, V, d) || check_act_dtype(act_dtype)) return 0;
    JointArgs a = make_args(nullptr, nullptr, nullptr, nullptr, nullptr, B, T, U, V, 0, d, U - 1, 0, 0.f);
    const bool tc = backward ? use_tc_bwd(tf32, a) : use_tc(tf32, a);
    return tr_workspace_bytes(a, node_capacity(B, T, U), tc, backward != 0, act_dtype);
}

int rnnt_forward_impl(const void* encoder, const void* decoder, int act_dtype, const float* joint_W,
                      const int32_t* targets, const int32_t* in_lens, const int32_t* tgt_lens, int B, int T, int U,
                      int V, int d, int S, int blank_idx, int tf32, float* loss, double* alpha, float* log_P_blank,
                      float* log_P_y, float* log_prob, void* workspace, size_t workspace_bytes, asr_stream_t stream,
                      void* stash = nullptr, size_t stash_bytes = 0) {
    NvtxRange range("asr::rnnt_forward");
    if (bad_dims(B, T, U, V, d) || S < 0 || blank_idx < 0 || blank_idx >= V || check_act_dtype(act_dtype))
        return ASR_ERR_INVALID_ARGUMENT;
    if (B == 0) return ASR_OK;
    if (!encoder || !decoder || !joint_W || !in_lens || !tgt_lens || !loss || !alpha || !log_P_blank || !log_P_y ||
        !log_prob || (S > 0 && !targets))
        return ASR_ERR_INVALID_ARGUMENT;
    if (U > kMaxLabelPositions) return ASR_ERR_UNSUPPORTED;
    JointArgs a = make_args(static_cast<const float*>(encoder), static_cast<const float*>(decoder), joint_W, nullptr,
                            targets, B, T, U, V, 0, d, S, blank_idx, 0.f);
    const int64_t cap = node_capacity(B, T, U);
    const bool tc = use_tc(tf32, a);
    if (!workspace || workspace_bytes < tr_workspace_bytes(a, cap, tc, false, act_dtype)) return ASR_ERR_WORKSPACE;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    TrWorkspace w = carve(workspace, a, cap, tc, false, act_dtype);
    a.m = w.meta;
    int rc = bind_activations(a, encoder, decoder, act_dtype, w, st);
    if (rc) return rc;
    rc = launch_lattice_prep(in_lens, tgt_lens, B, T, U, S, w.meta, st);
    if (rc) return rc;
    JointFwdOut o{log_P_blank, log_P_blank + cap, log_P_y, nullptr};
    rc = tc ? tc_joint_forward(a, o, (int)cap, w.joint, w.joint_bytes, st, stash_view(tf32, a, stash, stash_bytes))
            : simt_joint_forward(a, o, st);
    if (rc) return rc;
    return launch_rnnt_alpha(w.meta, B, U, log_P_blank, log_P_y, alpha, log_prob, loss, st);
}

int rnnt_backward_impl(const void* encoder, const void* decoder, int act_dtype, const float* joint_W,
                       const int32_t* targets, const int32_t* in_lens, const int32_t* tgt_lens, int B, int T, int U,
                       int V, int d, int S, int blank_idx, const double* alpha, const float* log_P_blank,
                       const float* log_P_y, const float* log_prob, const float* grad_loss, int tf32,
                       void* grad_encoder, void* grad_decoder, float* grad_joint_W, void* workspace,
                       size_t workspace_bytes, asr_stream_t stream, const void* stash = nullptr,
                       size_t stash_bytes = 0) {
    NvtxRange range("asr::rnnt_backward");
    if (bad_dims(B, T, U, V, d) || S < 0 || blank_idx < 0 || blank_idx >= V || check_act_dtype(act_dtype))
        return ASR_ERR_INVALID_ARGUMENT;
    if (!grad_joint_W) return ASR_ERR_INVALID_ARGUMENT;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (B == 0) {
        ASR_CUDA_TRY(cudaMemsetAsync(grad_joint_W, 0, sizeof(float) * (size_t)V * d, st));
        return ASR_OK;
    }
    if (!encoder || !decoder || !joint_W || !in_lens || !tgt_lens || !alpha || !log_P_blank || !log_P_y ||
        !log_prob || !grad_loss || !grad_encoder || !grad_decoder || (S > 0 && !targets))
        return ASR_ERR_INVALID_ARGUMENT;
    if (U > kMaxLabelPositions) return ASR_ERR_UNSUPPORTED;
    JointArgs a = make_args(static_cast<const float*>(encoder), static_cast<const float*>(decoder), joint_W, nullptr,
                            targets, B, T, U, V, 0, d, S, blank_idx, 0.f);
    const int64_t cap = node_capacity(B, T, U);
    const bool tc = use_tc_bwd(tf32, a);
    if (!workspace || workspace_bytes < tr_workspace_bytes(a, cap, tc, true, act_dtype)) return ASR_ERR_WORKSPACE;
    TrWorkspace w = carve(workspace, a, cap, tc, true, act_dtype);
    a.m = w.meta;
    int rc = bind_activations(a, encoder, decoder, act_dtype, w, st);
    if (rc) return rc;
    rc = launch_lattice_prep(in_lens, tgt_lens, B, T, U, S, w.meta, st);
    if (rc) return rc;
    rc = launch_rnnt_beta(w.meta, B, U, log_P_blank, log_P_y, alpha, grad_loss, w.cb, w.ct, w.beta, st);
    if (rc) return rc;
    float *ge, *gd;
    rc = zero_act_grads(a, w, grad_encoder, grad_decoder, &ge, &gd, st);
    if (rc) return rc;
    ASR_CUDA_TRY(cudaMemsetAsync(grad_joint_W, 0, sizeof(float) * (size_t)V * d, st));
    JointBwdIn in{log_P_blank + cap, w.cb, w.ct, nullptr};
    JointBwdOut o{ge, gd, grad_joint_W, nullptr};
    rc = tc ? tc_joint_backward(a, in, o, (int)cap, w.joint, w.joint_bytes, st, stash_view(tf32, a, stash, stash_bytes))
            : simt_joint_backward(a, in, o, (int)cap, w.joint, w.joint_bytes, st);
    if (rc) return rc;
    return finish_act_grads(a, w, grad_encoder, grad_decoder, st);
}

}  // namespace

extern "C" size_t asr_rnnt_workspace_bytes(int B, int T, int U, int V, int d, int tf32, int backward) {
    return rnnt_workspace_impl(B, T, U, V, d, tf32, backward, ASR_DTYPE_F32);
}

extern "C" size_t asr_rnnt_workspace_bytes_ex(int B, int T, int U, int V, int d, int tf32, int backward,
                                               int act_dtype) {
    return rnnt_workspace_impl(B, T, U, V, d, tf32, backward, act_dtype);
}

extern "C" int asr_rnnt_forward(const float* encoder, const float* decoder, const float* joint_W,
                                const int32_t* targets, const int32_t* in_lens, const int32_t* tgt_lens, int B,
                                int T, int U, int V, int d, int S, int blank_idx, int tf32, float* loss, double* alpha,
                                float* log_P_blank, float* log_P_y, float* log_prob, void* workspace,
                                size_t workspace_bytes, asr_stream_t stream) {
    return rnnt_forward_impl(encoder, decoder, ASR_DTYPE_F32, joint_W, targets, in_lens, tgt_lens, B, T, U, V, d, S,
                             blank_idx, tf32, loss, alpha, log_P_blank, log_P_y, log_prob, workspace,
                             workspace_bytes, stream);
}

extern "C" int asr_rnnt_forward_ex(const void* encoder, const void* decoder, int act_dtype, const float* joint_W,
                                   const int32_t* targets, const int32_t* in_lens, const int32_t* tgt_lens, int B,
                                   int T, int U, int V, int d, int S, int blank_idx, int tf32, float* loss,
                                   double* alpha, float* log_P_blank, float* log_P_y, float* log_prob,
                                   void* workspace, size_t workspace_bytes, asr_stream_t stream) {
    return rnnt_forward_impl(encoder, decoder, act_dtype, joint_W, targets, in_lens, tgt_lens, B, T, U, V, d, S,
                             blank_idx, tf32, loss, alpha, log_P_blank, log_P_y, log_prob, workspace,
                             workspace_bytes, stream);
}

extern "C" int asr_rnnt_backward(const float* encoder, const float* decoder, const float* joint_W,
                                 const int32_t* targets, const int32_t* in_lens, const int32_t* tgt_lens, int B,
                                 int T, int U, int V, int d, int S, int blank_idx, const double* alpha,
                                 const float* log_P_blank, const float* log_P_y, const float* log_prob,
                                 const float* grad_loss, int tf32, float* grad_encoder, float* grad_decoder,
                                 float* grad_joint_W, void* workspace, size_t workspace_bytes,
                                 asr_stream_t stream) {
    return rnnt_backward_impl(encoder, decoder, ASR_DTYPE_F32, joint_W, targets, in_lens, tgt_lens, B, T, U, V, d, S,
                              blank_idx, alpha, log_P_blank, log_P_y, log_prob, grad_loss, tf32, grad_encoder,
                              grad_decoder, grad_joint_W, workspace, workspace_bytes, stream);
}

extern "C" int asr_rnnt_backward_ex(const void* encoder, const void* decoder, int act_dtype, const float* joint_W,
                                    const int32_t* targets, const int32_t* in_lens, const int32_t* tgt_lens, int B,
                                    int T, int U, int V, int d, int S, int blank_idx, const double* alpha,
                                    const float* log_P_blank, const float* log_P_y, const float* log_prob,
                                    const float* grad_loss, int tf32, void* grad_encoder, void* grad_decoder,
                                    float* grad_joint_W, void* workspace, size_t workspace_bytes,
                                    asr_stream_t stream) {
    return rnnt_backward_impl(encoder, decoder, act_dtype, joint_W, targets, in_lens, tgt_lens, B, T, U, V, d, S,
                              blank_idx, alpha, log_P_blank, log_P_y, log_prob, grad_loss, tf32, grad_encoder,
                              grad_decoder, grad_joint_W, workspace, workspace_bytes, stream);
}

// -------------------------------------------------------------------------- TDT

namespace {
bool bad_tdt(int n_dur, int max_duration) {
    return n_dur < 1 || n_dur > kTdtMaxDurClasses || max_duration < 1 || max_duration > kTdtMaxDuration;
}
}  // namespace

namespace {

size_t tdt_workspace_impl(int B, int T, int U, int V, int n_dur, int d, int tf32, int backward, int act_dtype) {
    if (bad_dims(B, T, U, V, d) || n_dur < 1 || check_act_dtype(act_dtype)) return 0;
    JointArgs a = make_args(nullptr, nullptr, nullptr, nullptr, nullptr, B, T, U, V, n_dur, d, U - 1, 0, 0.f);
    const bool tc = backward ? use_tc_bwd(tf32, a) : use_tc(tf32, a);
    return tr_workspace_bytes(a, node_capacity(B, T, U), tc, backward != 0, act_dtype);
}

int tdt_forward_impl(const void* encoder, const void* decoder, int act_dtype, const float* joint_W,
                     const float* joint_W_dur, const int32_t* targets, const int32_t* in_lens, const int32_t* tgt_lens,
                     const int32_t* durations, int n_dur, int max_duration, int has_zero, int B, int T, int U, int V,
                     int d, int S, int blank_idx, float sigma, int tf32, float* loss, double* alpha,
                     float* log_P_blank, float* log_P_y, float* log_P_dur, float* log_prob, void* workspace,
                     size_t workspace_bytes, asr_stream_t stream, void* stash = nullptr, size_t stash_bytes = 0) {
    NvtxRange range("asr::tdt_forward");
    if (bad_dims(B, T, U, V, d) || S < 0 || blank_idx < 0 || blank_idx >= V || bad_tdt(n_dur, max_duration) ||
        check_act_dtype(act_dtype))
        return ASR_ERR_INVALID_ARGUMENT;
    if (B == 0) return ASR_OK;
    if (!encoder || !decoder || !joint_W || !joint_W_dur || !durations || !in_lens || !tgt_lens || !loss ||
        !alpha || !log_P_blank || !log_P_y || !log_P_dur || !log_prob || (S > 0 && !targets))
        return ASR_ERR_INVALID_ARGUMENT;
    if (U > kMaxLabelPositions) return ASR_ERR_UNSUPPORTED;
    JointArgs a = make_args(static_cast<const float*>(encoder), static_cast<const float*>(decoder), joint_W,
                            joint_W_dur, targets, B, T, U, V, n_dur, d, S, blank_idx, sigma);
    const int64_t cap = node_capacity(B, T, U);
    const bool tc = use_tc(tf32, a);
    if (!workspace || workspace_bytes < tr_workspace_bytes(a, cap, tc, false, act_dtype)) return ASR_ERR_WORKSPACE;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    TrWorkspace w = carve(workspace, a, cap, tc, false, act_dtype);
    a.m = w.meta;
    int rc = bind_activations(a, encoder, decoder, act_dtype, w, st);
    if (rc) return rc;
    rc = launch_lattice_prep(in_lens, tgt_lens, B, T, U, S, w.meta, st);
    if (rc) return rc;
    JointFwdOut o{log_P_blank, log_P_blank + cap, log_P_y, log_P_dur};
    rc = tc ? tc_joint_forward(a, o, (int)cap, w.joint, w.joint_bytes, st, stash_view(tf32, a, stash, stash_bytes))
            : simt_joint_forward(a, o, st);
    if (rc) return rc;
    return launch_tdt_alpha(w.meta, B, U, max_duration, durations, n_dur, has_zero, log_P_blank, log_P_y, log_P_dur,
                            alpha, log_prob, loss, st);
}

int tdt_backward_impl(const void* encoder, const void* decoder, int act_dtype, const float* joint_W,
                      const float* joint_W_dur, const int32_t* targets, const int32_t* in_lens,
                      const int32_t* tgt_lens, const int32_t* durations, int n_dur, int max_duration, int has_zero,
                      int B, int T, int U, int V, int d, int S, int blank_idx, const double* alpha,
                      const float* log_P_blank, const float* log_P_y, const float* log_P_dur, const float* log_prob,
                      const float* grad_loss, int tf32, void* grad_encoder, void* grad_decoder, float* grad_joint_W,
                      float* grad_joint_W_dur, void* workspace, size_t workspace_bytes, asr_stream_t stream,
                      const void* stash = nullptr, size_t stash_bytes = 0) {
    NvtxRange range("asr::tdt_backward");
    if (bad_dims(B, T, U, V, d) || S < 0 || blank_idx < 0 || blank_idx >= V || bad_tdt(n_dur, max_duration) ||
        check_act_dtype(act_dtype))
        return ASR_ERR_INVALID_ARGUMENT;
    if (!grad_joint_W || !grad_joint_W_dur) return ASR_ERR_INVALID_ARGUMENT;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (B == 0) {
        ASR_CUDA_TRY(cudaMemsetAsync(grad_joint_W, 0, sizeof(float) * (size_t)V * d, st));
        ASR_CUDA_TRY(cudaMemsetAsync(grad_joint_W_dur, 0, sizeof(float) * (size_t)n_dur * d, st));
        return ASR_OK;
    }
    if (!encoder || !decoder || !joint_W || !joint_W_dur || !durations || !in_lens || !tgt_lens || !alpha ||
        !log_P_blank || !log_P_y || !log_P_dur || !log_prob || !grad_loss || !grad_encoder || !grad_decoder ||
        (S > 0 && !targets))
        return ASR_ERR_INVALID_ARGUMENT;
    if (U > kMaxLabelPositions) return ASR_ERR_UNSUPPORTED;
    JointArgs a = make_args(static_cast<const float*>(encoder), static_cast<const float*>(decoder), joint_W,
                            joint_W_dur, targets, B, T, U, V, n_dur, d, S, blank_idx, 0.f);
    const int64_t cap = node_capacity(B, T, U);
    const bool tc = use_tc_bwd(tf32, a);
    if (!workspace || workspace_bytes < tr_workspace_bytes(a, cap, tc, true, act_dtype)) return ASR_ERR_WORKSPACE;
    TrWorkspace w = carve(workspace, a, cap, tc, true, act_dtype);
    a.m = w.meta;
    int rc = bind_activations(a, encoder, decoder, act_dtype, w, st);
    if (rc) return rc;
    rc = launch_lattice_prep(in_lens, tgt_lens, B, T, U, S, w.meta, st);
    if (rc) return rc;
    rc = launch_tdt_beta(w.meta, B, U, max_duration, durations, n_dur, has_zero, log_P_blank, log_P_y, log_P_dur,
                         alpha, grad_loss, w.cb, w.ct, w.gdur, w.beta, st);
    if (rc) return rc;
    float *ge, *gd;
    rc = zero_act_grads(a, w, grad_encoder, grad_decoder, &ge, &gd, st);
    if (rc) return rc;
    ASR_CUDA_TRY(cudaMemsetAsync(grad_joint_W, 0, sizeof(float) * (size_t)V * d, st));
    ASR_CUDA_TRY(cudaMemsetAsync(grad_joint_W_dur, 0, sizeof(float) * (size_t)n_dur * d, st));
    JointBwdIn in{log_P_blank + cap, w.cb, w.ct, w.gdur};
    JointBwdOut o{ge, gd, grad_joint_W, grad_joint_W_dur};
    rc = tc ? tc_joint_backward(a, in, o, (int)cap, w.joint, w.joint_bytes, st, stash_view(tf32, a, stash, stash_bytes))
            : simt_joint_backward(a, in, o, (int)cap, w.joint, w.joint_bytes, st);
    if (rc) return rc;
    return finish_act_grads(a, w, grad_encoder, grad_decoder, st);
}

}  // namespace

extern "C" size_t asr_tdt_workspace_bytes(int B, int T, int U, int V, int n_dur, int d, int tf32, int backward) {
    return tdt_workspace_impl(B, T, U, V, n_dur, d, tf32, backward, ASR_DTYPE_F32);
}

extern "C" size_t asr_tdt_workspace_bytes_ex(int B, int T, int U, int V, int n_dur, int d, int tf32, int backward,
                                              int act_dtype) {
    return tdt_workspace_impl(B, T, U, V, n_dur, d, tf32, backward, act_dtype);
}

extern "C" int asr_tdt_forward(const float* encoder, const float* decoder, const float* joint_W,
                               const float* joint_W_dur, const int32_t* targets, const int32_t* in_lens,
                               const int32_t* tgt_lens, const int32_t* durations, int n_dur, int max_duration,
                               int has_zero, int B, int T, int U, int V, int d, int S, int blank_idx, float sigma,
                               int tf32, float* loss, double* alpha, float* log_P_blank, float* log_P_y,
                               float* log_P_dur, float* log_prob, void* workspace, size_t workspace_bytes,
                               asr_stream_t stream) {
    return tdt_forward_impl(encoder, decoder, ASR_DTYPE_F32, joint_W, joint_W_dur, targets, in_lens, tgt_lens,
                            durations, n_dur, max_duration, has_zero, B, T, U, V, d, S, blank_idx, sigma, tf32, loss,
                            alpha, log_P_blank, log_P_y, log_P_dur, log_prob, workspace, workspace_bytes, stream);
}

extern "C" int asr_tdt_forward_ex(const void* encoder, const void* decoder, int act_dtype, const float* joint_W,
                                  const float* joint_W_dur, const int32_t* targets, const int32_t* in_lens,
                                  const int32_t* tgt_lens, const int32_t* durations, int n_dur, int max_duration,
                                  int has_zero, int B, int T, int U, int V, int d, int S, int blank_idx, float sigma,
                                  int tf32, float* loss, double* alpha, float* log_P_blank, float* log_P_y,
                                  float* log_P_dur, float* log_prob, void* workspace, size_t workspace_bytes,
                                  asr_stream_t stream) {
    return tdt_forward_impl(encoder, decoder, act_dtype, joint_W, joint_W_dur, targets, in_lens, tgt_lens, durations,
                            n_dur, max_duration, has_zero, B, T, U, V, d, S, blank_idx, sigma, tf32, loss, alpha,
                            log_P_blank, log_P_y, log_P_dur, log_prob, workspace, workspace_bytes, stream);
}

extern "C" int asr_tdt_backward(const float* encoder, const float* decoder, const float* joint_W,
                                const float* joint_W_dur, const int32_t* targets, const int32_t* in_lens,
                                const int32_t* tgt_lens, const int32_t* durations, int n_dur, int max_duration,
                                int has_zero, int B, int T, int U, int V, int d, int S, int blank_idx,
                                const double* alpha, const float* log_P_blank, const float* log_P_y,
                                const float* log_P_dur, const float* log_prob, const float* grad_loss, int tf32,
                                float* grad_encoder, float* grad_decoder, float* grad_joint_W,
                                float* grad_joint_W_dur, void* workspace, size_t workspace_bytes,
                                asr_stream_t stream) {
    return tdt_backward_impl(encoder, decoder, ASR_DTYPE_F32, joint_W, joint_W_dur, targets, in_lens, tgt_lens,
                             durations, n_dur, max_duration, has_zero, B, T, U, V, d, S, blank_idx, alpha,
                             log_P_blank, log_P_y, log_P_dur, log_prob, grad_loss, tf32, grad_encoder, grad_decoder,
                             grad_joint_W, grad_joint_W_dur, workspace, workspace_bytes, stream);
}

extern "C" int asr_tdt_backward_ex(const void* encoder, const void* decoder, int act_dtype, const float* joint_W,
                                   const float* joint_W_dur, const int32_t* targets, const int32_t* in_lens,
                                   const int32_t* tgt_lens, const int32_t* durations, int n_dur, int max_duration,
                                   int has_zero, int B, int T, int U, int V, int d, int S, int blank_idx,
                                   const double* alpha, const float* log_P_blank, const float* log_P_y,
                                   const float* log_P_dur, const float* log_prob, const float* grad_loss, int tf32,
                                   void* grad_encoder, void* grad_decoder, float* grad_joint_W,
                                   float* grad_joint_W_dur, void* workspace, size_t workspace_bytes,
                                   asr_stream_t stream) {
    return tdt_backward_impl(encoder, decoder, act_dtype, joint_W, joint_W_dur, targets, in_lens, tgt_lens,
                             durations, n_dur, max_duration, has_zero, B, T, U, V, d, S, blank_idx, alpha,
                             log_P_blank, log_P_y, log_P_dur, log_prob, grad_loss, tf32, grad_encoder, grad_decoder,
                             grad_joint_W, grad_joint_W_dur, workspace, workspace_bytes, stream);
}

// ------------------------------------------------------------------ diagnostics

extern "C" int asr_workspace_status(const void* workspace, int B, int* clamped, asr_stream_t stream) {
    if (!workspace || !clamped || B < 1) return ASR_ERR_INVALID_ARGUMENT;
    LatticeMeta m;
    char* p = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255));
    lattice_meta_carve(p, B, &m);
    int32_t v = 0;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    ASR_CUDA_TRY(cudaMemcpyAsync(&v, m.status, sizeof(int32_t), cudaMemcpyDeviceToHost, st));
    ASR_CUDA_TRY(cudaStreamSynchronize(st));
    *clamped = v;
    return ASR_OK;
}

// ------------------------------------------------------------------ logit stash

extern "C" size_t asr_logit_stash_bytes(int B, int T, int U, int V, int n_dur, int d, int tf32) {
    if (bad_dims(B, T, U, V, d) || n_dur < 0 || B == 0) return 0;
    JointArgs a = make_args(nullptr, nullptr, nullptr, nullptr, nullptr, B, T, U, V, n_dur, d, U - 1, 0, 0.f);
    if (!use_tc_bwd(tf32, a)) return 0;
    const int64_t nodes = (node_capacity(B, T, U) + 255) / 256 * 256;
    return (size_t)nodes * tc_stash_bytes_per_node(a) + 512;
}

extern "C" int asr_rnnt_forward_stash(const void* encoder, const void* decoder, int act_dtype, const float* joint_W,
                                      const int32_t* targets, const int32_t* in_lens, const int32_t* tgt_lens, int B,
                                      int T, int U, int V, int d, int S, int blank_idx, int tf32, float* loss,
                                      double* alpha, float* log_P_blank, float* log_P_y, float* log_prob,
                                      void* stash, size_t stash_bytes, void* workspace, size_t workspace_bytes,
                                      asr_stream_t stream) {
    return rnnt_forward_impl(encoder, decoder, act_dtype, joint_W, targets, in_lens, tgt_lens, B, T, U, V, d, S,
                             blank_idx, tf32, loss, alpha, log_P_blank, log_P_y, log_prob, workspace,
                             workspace_bytes, stream, stash, stash_bytes);
}

extern "C" int asr_rnnt_backward_stash(const void* encoder, const void* decoder, int act_dtype,
                                       const float* joint_W, const int32_t* targets, const int32_t* in_lens,
                                       const int32_t* tgt_lens, int B, int T, int U, int V, int d, int S,
                                       int blank_idx, const double* alpha, const float* log_P_blank,
                                       const float* log_P_y, const float* log_prob, const float* grad_loss, int tf32,
                                       void* grad_encoder, void* grad_decoder, float* grad_joint_W,
                                       const void* stash, size_t stash_bytes, void* workspace,
                                       size_t workspace_bytes, asr_stream_t stream) {
    return rnnt_backward_impl(encoder, decoder, act_dtype, joint_W, targets, in_lens, tgt_lens, B, T, U, V, d, S,
                              blank_idx, alpha, log_P_blank, log_P_y, log_prob, grad_loss, tf32, grad_encoder,
                              grad_decoder, grad_joint_W, workspace, workspace_bytes, stream, stash, stash_bytes);
}

extern "C" int asr_tdt_forward_stash(const void* encoder, const void* decoder, int act_dtype, const float* joint_W,
                                     const float* joint_W_dur, const int32_t* targets, const int32_t* in_lens,
                                     const int32_t* tgt_lens, const int32_t* durations, int n_dur, int max_duration,
                                     int has_zero, int B, int T, int U, int V, int d, int S, int blank_idx,
                                     float sigma, int tf32, float* loss, double* alpha, float* log_P_blank,
                                     float* log_P_y, float* log_P_dur, float* log_prob, void* stash,
                                     size_t stash_bytes, void* workspace, size_t workspace_bytes,
                                     asr_stream_t stream) {
    return tdt_forward_impl(encoder, decoder, act_dtype, joint_W, joint_W_dur, targets, in_lens, tgt_lens, durations,
                            n_dur, max_duration, has_zero, B, T, U, V, d, S, blank_idx, sigma, tf32, loss, alpha,
                            log_P_blank, log_P_y, log_P_dur, log_prob, workspace, workspace_bytes, stream, stash,
                            stash_bytes);
}

extern "C" int asr_tdt_backward_stash(const void* encoder, const void* decoder, int act_dtype, const float* joint_W,
                                      const float* joint_W_dur, const int32_t* targets, const int32_t* in_lens,
                                      const int32_t* tgt_lens, const int32_t* durations, int n_dur,
                                      int max_duration, int has_zero, int B, int T, int U, int V, int d, int S,
                                      int blank_idx, const double* alpha, const float* log_P_blank,
                                      const float* log_P_y, const float* log_P_dur, const float* log_prob,
                                      const float* grad_loss, int tf32, void* grad_encoder, void* grad_decoder,
                                      float* grad_joint_W, float* grad_joint_W_dur, const void* stash,
                                      size_t stash_bytes, void* workspace, size_t workspace_bytes,
                                      asr_stream_t stream) {
    return tdt_backward_impl(encoder, decoder, act_dtype, joint_W, joint_W_dur, targets, in_lens, tgt_lens, durations,
                             n_dur, max_duration, has_zero, B, T, U, V, d, S, blank_idx, alpha, log_P_blank, log_P_y,
                             log_P_dur, log_prob, grad_loss, tf32, grad_encoder, grad_decoder, grad_joint_W,
                             grad_joint_W_dur, workspace, workspace_bytes, stream, stash, stash_bytes);
}
