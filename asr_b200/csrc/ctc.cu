// CTC forward (alpha) and backward (beta fused with d loss / d logits).
//
// One CTA of up to 8 warps per utterance: the 2S+1 extended-label states are
// split into thread-contiguous blocks of KS (about two) states held in
// registers. The stay / advance / skip moves (ctc.cu:84-98 of the reference)
// need the two states just left of a block (right, for beta): inside a warp they
// come by shuffle, across warps through shared memory, so a time step is a few
// register ops, two shuffles and one CTA barrier, with the next step's emission
// log-probs (and, for beta, alpha) prefetched meanwhile. The backward scatters
// state posteriors into a shared-memory row of V bins (the blank states' mass
// summed per warp first; two rows, by step parity) and writes each gradient row
// once, one step later, in the same block as the recursion.
#include "common.cuh"

namespace asr {
namespace {

// log(exp(a) + exp(b) + exp(c)) with float64 state and an fp32 correction term.
__device__ __forceinline__ double lse3_d(double a, double b, double c) {
    const double m = fmax(a, fmax(b, c));
    if (m == -INFINITY) return -INFINITY;
    return m + (double)__logf(__expf((float)(a - m)) + __expf((float)(b - m)) + __expf((float)(c - m)));
}

struct CtcUtt {
    int Tb, Sb, L;
};

__device__ __forceinline__ CtcUtt ctc_utt(const int32_t* in_lens, const int32_t* tgt_lens, int b, int T, int S) {
    CtcUtt u;
    u.Tb = min(max(in_lens[b], 1), T);
    u.Sb = min(max(tgt_lens[b], 0), S);
    u.L = 2 * u.Sb + 1;
    return u;
}

// log Z from the last blank and last label state (ctc.cu:106-113).
__device__ __forceinline__ double ctc_logz(double last, double prev, int L) {
    if (L == 1) return last;
    const double m = fmax(last, prev);
    if (m == -INFINITY) return -INFINITY;
    return m + (double)log1pf(__expf((float)(fmin(last, prev) - m)));
}

// The forward variable is float64: on T ~ 10^2..10^3 frames |alpha| reaches 10^3,
// where fp32 rounding along the recursion would cost ~1e-3 in the posteriors.
//
// One CTA of NW warps per utterance, KS consecutive states per thread. The two
// states left of a warp's first thread (for the stay / advance / skip moves) come
// from the previous warp through shared memory, double-buffered by step parity so
// one barrier per step suffices; inside a warp they come by shuffle.
template <int KS, int NW>
__global__ void __launch_bounds__(32 * NW)
    ctc_alpha_kernel(const float* __restrict__ lp, const int32_t* __restrict__ targets,
                     const int32_t* __restrict__ in_lens, const int32_t* __restrict__ tgt_lens, int B, int T, int V,
                     int S, double* __restrict__ alpha, float* __restrict__ log_Z) {
    __shared__ double bnd[2][NW][2];  // last two states of each warp (previous step)
    __shared__ double fin[2];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = threadIdx.x;
    const int b = blockIdx.x;
    const CtcUtt ut = ctc_utt(in_lens, tgt_lens, b, T, S);
    const int Lmax = 2 * S + 1;
    const int32_t* y = targets + (int64_t)b * S;
    const float* lpb = lp + (int64_t)b * T * V;
    double* ab = alpha + (int64_t)b * T * Lmax;

    int lab[KS];
    bool skip[KS], in[KS];
#pragma unroll
    for (int j = 0; j < KS; ++j) {
        const int s = g * KS + j;
        in[j] = s < ut.L;
        const bool odd = s & 1;
        lab[j] = (odd && in[j]) ? y[s >> 1] : 0;
        skip[j] = in[j] && odd && (s >> 1) > 0 && y[s >> 1] != y[(s >> 1) - 1];
    }
    double a[KS];
    float nxt[KS];
#pragma unroll
    for (int j = 0; j < KS; ++j) {
        const int s = g * KS + j;
        a[j] = (in[j] && s <= 1) ? (double)lpb[lab[j]] : -INFINITY;
        if (in[j]) ab[s] = a[j];
        nxt[j] = (in[j] && ut.Tb > 1) ? lpb[V + lab[j]] : 0.f;
    }
    for (int t = 1; t < ut.Tb; ++t) {
        float cur[KS];
#pragma unroll
        for (int j = 0; j < KS; ++j) cur[j] = nxt[j];
        if (t + 1 < ut.Tb) {
#pragma unroll
            for (int j = 0; j < KS; ++j) nxt[j] = in[j] ? lpb[(int64_t)(t + 1) * V + lab[j]] : 0.f;
        }
        // publish this warp's last two states, then gather the two states left of each block
        const double e1 = __shfl_sync(0xffffffffu, a[KS - 1], 31);
        const double e2 = KS >= 2 ? __shfl_sync(0xffffffffu, a[KS >= 2 ? KS - 2 : 0], 31)
                                  : __shfl_sync(0xffffffffu, a[0], 30);
        if (NW > 1 && lane == 0) {
            bnd[t & 1][warp][0] = e1;
            bnd[t & 1][warp][1] = e2;
        }
        if (NW > 1) __syncthreads();
        double x1 = __shfl_up_sync(0xffffffffu, a[KS - 1], 1);
        double x2 = (KS >= 2) ? __shfl_up_sync(0xffffffffu, a[KS >= 2 ? KS - 2 : 0], 1)
                              : __shfl_up_sync(0xffffffffu, a[0], 2);
        const double p1 = (NW > 1 && warp > 0) ? bnd[t & 1][warp > 0 ? warp - 1 : 0][0] : -INFINITY;
        const double p2 = (NW > 1 && warp > 0) ? bnd[t & 1][warp > 0 ? warp - 1 : 0][1] : -INFINITY;
        if (lane == 0) {
            x1 = p1;
            x2 = p2;
        }
        if (KS == 1 && lane == 1) x2 = p1;
        double na[KS];
#pragma unroll
        for (int j = 0; j < KS; ++j) {
            const double q1 = (j >= 1) ? a[j >= 1 ? j - 1 : 0] : x1;
            const double q2 = (j >= 2) ? a[j >= 2 ? j - 2 : 0] : (j == 1 ? x1 : x2);
            na[j] = in[j] ? lse3_d(a[j], q1, skip[j] ? q2 : -INFINITY) + cur[j] : -INFINITY;
        }
#pragma unroll
        for (int j = 0; j < KS; ++j) {
            a[j] = na[j];
            if (in[j]) ab[(int64_t)t * Lmax + g * KS + j] = a[j];
        }
    }
#pragma unroll
    for (int j = 0; j < KS; ++j) {
        const int s = g * KS + j;
        if (s == ut.L - 1) fin[0] = a[j];
        if (s == ut.L - 2) fin[1] = a[j];
    }
    __syncthreads();
    if (g == 0) log_Z[b] = (float)ctc_logz(fin[0], ut.L >= 2 ? fin[1] : -INFINITY, ut.L);
}

template <int KS, int NW>
__global__ void __launch_bounds__(32 * NW)
    ctc_grad_kernel(const double* __restrict__ alpha, const float* __restrict__ lp,
                    const int32_t* __restrict__ targets, const int32_t* __restrict__ in_lens,
                    const int32_t* __restrict__ tgt_lens, const float* __restrict__ grad_loss, int zero_infinity,
                    int post_only, int B, int T, int V, int S, float* __restrict__ grad) {
    extern __shared__ float row[];     // (2, V) posterior mass per column, by step parity
    __shared__ double bnd[2][NW][2];   // first two states of each warp (beta + emission)
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = threadIdx.x;
    const int b = blockIdx.x;
    const CtcUtt ut = ctc_utt(in_lens, tgt_lens, b, T, S);
    const int Lmax = 2 * S + 1;
    const int32_t* y = targets + (int64_t)b * S;
    const float* lpb = lp + (int64_t)b * T * V;
    const double* ab = alpha + (int64_t)b * T * Lmax;
    float* gb = grad + (int64_t)b * T * V;
    // log Z in float64, from the stored forward variable
    const double* alast = ab + (int64_t)(ut.Tb - 1) * Lmax;
    const double logZ = ctc_logz(alast[ut.L - 1], ut.L >= 2 ? alast[ut.L - 2] : -INFINITY, ut.L);
    const float gl = grad_loss[b];

    const bool dead = zero_infinity && !isfinite(logZ);
    // rows the recursion never reaches are zero (the reference zero-initialises)
    for (int64_t i = (int64_t)(dead ? 0 : ut.Tb) * V + g; i < (int64_t)T * V; i += blockDim.x) gb[i] = 0.f;
    if (dead) return;
    for (int v = g; v < 2 * V; v += blockDim.x) row[v] = 0.f;

    int lab[KS];
    bool skip[KS], in[KS];
#pragma unroll
    for (int j = 0; j < KS; ++j) {
        const int s = g * KS + j;
        in[j] = s < ut.L;
        const bool odd = s & 1;
        lab[j] = (odd && in[j]) ? y[s >> 1] : 0;
        // skip move s -> s+2 allowed when labels differ (ctc.cu:183-185)
        skip[j] = in[j] && odd && (s >> 1) < ut.Sb - 1 && y[s >> 1] != y[(s >> 1) + 1];
    }
    // beta at t = T_b - 1 excludes the emission at t (ctc.cu:137-146)
    double be[KS];
#pragma unroll
    for (int j = 0; j < KS; ++j) {
        const int s = g * KS + j;
        be[j] = (in[j] && (s == ut.L - 1 || s == ut.L - 2)) ? 0.0 : -INFINITY;
    }
    float lpt[KS];
    double acur[KS];  // alpha of the current step, loaded one step ahead
#pragma unroll
    for (int j = 0; j < KS; ++j) {
        lpt[j] = in[j] ? lpb[(int64_t)(ut.Tb - 1) * V + lab[j]] : 0.f;
        acur[j] = in[j] ? ab[(int64_t)(ut.Tb - 1) * Lmax + g * KS + j] : -INFINITY;
    }
    // Step t: publish the recursion's boundary states, one barrier, then in one
    // block (so their latencies overlap) the recursion to beta(t - 1), the state
    // posteriors of step t scattered into the row buffer of parity t, and the
    // gradient row of step t + 1, whose buffer every thread finished filling
    // before the barrier.
    auto write_row = [&](int tr) {
        float* rw = row + (tr & 1) * V;
        for (int v = g; v < V; v += blockDim.x) {
            const int64_t idx = (int64_t)tr * V + v;
            // post_only: the posterior mass per column only (the fused CTC head adds
            // the softmax part inside its joint kernel)
            gb[idx] = post_only ? gl * rw[v] : gl * (__expf(lpb[idx]) - rw[v]);
            rw[v] = 0.f;
        }
    };
    for (int t = ut.Tb - 1; t >= 0; --t) {
        // beta recursion (ctc.cu:180-204): c[s] = beta[s] + lp[t][lab(s)]
        double c[KS];
#pragma unroll
        for (int j = 0; j < KS; ++j) c[j] = in[j] ? be[j] + lpt[j] : -INFINITY;
        const double f1 = __shfl_sync(0xffffffffu, c[0], 0);
        const double f2 = KS >= 2 ? __shfl_sync(0xffffffffu, c[KS >= 2 ? 1 : 0], 0) : __shfl_sync(0xffffffffu, c[0], 1);
        if (NW > 1 && lane == 0) {
            bnd[t & 1][warp][0] = f1;
            bnd[t & 1][warp][1] = f2;
        }
        __syncthreads();  // boundary states published; the row of step t + 1 is complete
        // state posteriors of step t (ctc.cu:152-165)
        float post[KS];
#pragma unroll
        for (int j = 0; j < KS; ++j) post[j] = in[j] ? __expf((float)(acur[j] + be[j] - logZ)) : 0.f;
        // next step's alpha and emissions, in flight during the rest of the step
        float lnx[KS];
        if (t > 0) {
#pragma unroll
            for (int j = 0; j < KS; ++j) {
                if (in[j]) acur[j] = ab[(int64_t)(t - 1) * Lmax + g * KS + j];
                lnx[j] = in[j] ? lpb[(int64_t)(t - 1) * V + lab[j]] : 0.f;
            }
            double r1 = __shfl_down_sync(0xffffffffu, c[0], 1);
            double r2 = (KS >= 2) ? __shfl_down_sync(0xffffffffu, c[KS >= 2 ? 1 : 0], 1)
                                  : __shfl_down_sync(0xffffffffu, c[0], 2);
            const double n1 = (NW > 1 && warp + 1 < NW) ? bnd[t & 1][warp + 1 < NW ? warp + 1 : 0][0] : -INFINITY;
            const double n2 = (NW > 1 && warp + 1 < NW) ? bnd[t & 1][warp + 1 < NW ? warp + 1 : 0][1] : -INFINITY;
            if (lane == 31) {
                r1 = n1;
                r2 = n2;
            }
            if (KS == 1 && lane == 30) r2 = n1;
#pragma unroll
            for (int j = 0; j < KS; ++j) {
                const double q1 = (j + 1 < KS) ? c[j + 1 < KS ? j + 1 : 0] : r1;
                const double q2 = (j + 2 < KS) ? c[j + 2 < KS ? j + 2 : 0] : (j + 1 < KS ? r1 : r2);
                be[j] = in[j] ? lse3_d(c[j], q1, skip[j] ? q2 : -INFINITY) : -INFINITY;
            }
#pragma unroll
            for (int j = 0; j < KS; ++j) lpt[j] = lnx[j];
        }
        // the blank states (every even s, about half of them) share bin 0, so their
        // mass is summed over the warp first instead of contending for one address
        float* rw = row + (t & 1) * V;
        float pblank = 0.f;
#pragma unroll
        for (int j = 0; j < KS; ++j) {
            if (in[j]) {
                if ((g * KS + j) & 1)
                    atomicAdd(rw + lab[j], post[j]);
                else
                    pblank += post[j];
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) pblank += __shfl_xor_sync(0xffffffffu, pblank, o);
        if (lane == 0) atomicAdd(rw, pblank);
        if (t + 1 < ut.Tb) write_row(t + 1);
    }
    __syncthreads();  // the row of step 0 is complete
    write_row(0);
}

template <int KS, int NW>
int launch_ctc_alpha(const float* lp, const int32_t* tg, const int32_t* il, const int32_t* tl, int B, int T, int V,
                     int S, double* alpha, float* logz, cudaStream_t st) {
    KernelTimer kt("ctc_alpha", st);
    ctc_alpha_kernel<KS, NW><<<B, 32 * NW, 0, st>>>(lp, tg, il, tl, B, T, V, S, alpha, logz);
    ASR_LAUNCH_CHECK();
    return ASR_OK;
}

template <int KS, int NW>
int launch_ctc_grad(const double* alpha, const float* lp, const int32_t* tg, const int32_t* il, const int32_t* tl,
                    const float* gl, int zinf, int post_only, int B, int T, int V, int S, float* grad,
                    cudaStream_t st) {
    const size_t smem = 2 * sizeof(float) * (size_t)V;
    if (smem > 48 * 1024) {
        if (cudaFuncSetAttribute(ctc_grad_kernel<KS, NW>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
            cudaSuccess)
            return ASR_ERR_UNSUPPORTED;
    }
    KernelTimer kt("ctc_beta_grad", st);
    ctc_grad_kernel<KS, NW><<<B, 32 * NW, smem, st>>>(alpha, lp, tg, il, tl, gl, zinf, post_only, B, T, V, S, grad);
    ASR_LAUNCH_CHECK();
    return ASR_OK;
}

// (KS states per thread, NW warps per utterance) for L = 2S + 1 states: about two
// states per thread, up to 8 warps, then more states per thread; the longest
// targets (L up to 8192, S up to 4095 labels) take 16 warps of 16 states.
int ctc_shape(int S) {
    const int L = 2 * S + 1;
    if (L <= 32) return 11;
    if (L <= 64) return 21;
    if (L <= 128) return 22;
    if (L <= 256) return 24;
    if (L <= 512) return 28;
    if (L <= 1024) return 48;
    if (L <= 2048) return 88;
    if (L <= 4096) return 168;
    if (L <= 8192) return 1616;
    return 0;
}

}  // namespace
}  // namespace asr

using namespace asr;

extern "C" int asr_ctc_alpha(const float* log_probs, const int32_t* targets, const int32_t* in_lens,
                             const int32_t* tgt_lens, int B, int T, int V, int S, double* alpha, float* log_Z,
                             asr_stream_t stream) {
    NvtxRange range("asr::ctc_alpha");
    if (B < 0 || T < 1 || V < 1 || S < 0) return ASR_ERR_INVALID_ARGUMENT;
    if (B == 0) return ASR_OK;
    if (!log_probs || !in_lens || !tgt_lens || !alpha || !log_Z || (S > 0 && !targets)) return ASR_ERR_INVALID_ARGUMENT;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    switch (ctc_shape(S)) {
        case 11: return launch_ctc_alpha<1, 1>(log_probs, targets, in_lens, tgt_lens, B, T, V, S, alpha, log_Z, st);
        case 21: return launch_ctc_alpha<2, 1>(log_probs, targets, in_lens, tgt_lens, B, T, V, S, alpha, log_Z, st);
        case 22: return launch_ctc_alpha<2, 2>(log_probs, targets, in_lens, tgt_lens, B, T, V, S, alpha, log_Z, st);
        case 24: return launch_ctc_alpha<2, 4>(log_probs, targets, in_lens, tgt_lens, B, T, V, S, alpha, log_Z, st);
        case 28: return launch_ctc_alpha<2, 8>(log_probs, targets, in_lens, tgt_lens, B, T, V, S, alpha, log_Z, st);
        case 48: return launch_ctc_alpha<4, 8>(log_probs, targets, in_lens, tgt_lens, B, T, V, S, alpha, log_Z, st);
        case 88: return launch_ctc_alpha<8, 8>(log_probs, targets, in_lens, tgt_lens, B, T, V, S, alpha, log_Z, st);
        case 168: return launch_ctc_alpha<16, 8>(log_probs, targets, in_lens, tgt_lens, B, T, V, S, alpha, log_Z, st);
        case 1616:
            return launch_ctc_alpha<16, 16>(log_probs, targets, in_lens, tgt_lens, B, T, V, S, alpha, log_Z, st);
        default: return ASR_ERR_UNSUPPORTED;
    }
}

namespace asr {

int ctc_grad_dispatch(const double* alpha, const float* log_probs, const int32_t* targets, const int32_t* in_lens,
                      const int32_t* tgt_lens, const float* grad_loss, int zero_infinity, int post_only, int B, int T,
                      int V, int S, float* grad, cudaStream_t st) {
    const int z = zero_infinity ? 1 : 0;
    const int p = post_only ? 1 : 0;
    switch (ctc_shape(S)) {
        case 11: return launch_ctc_grad<1, 1>(alpha, log_probs, targets, in_lens, tgt_lens, grad_loss, z, p, B, T, V, S, grad, st);
        case 21: return launch_ctc_grad<2, 1>(alpha, log_probs, targets, in_lens, tgt_lens, grad_loss, z, p, B, T, V, S, grad, st);
        case 22: return launch_ctc_grad<2, 2>(alpha, log_probs, targets, in_lens, tgt_lens, grad_loss, z, p, B, T, V, S, grad, st);
        case 24: return launch_ctc_grad<2, 4>(alpha, log_probs, targets, in_lens, tgt_lens, grad_loss, z, p, B, T, V, S, grad, st);
        case 28: return launch_ctc_grad<2, 8>(alpha, log_probs, targets, in_lens, tgt_lens, grad_loss, z, p, B, T, V, S, grad, st);
        case 48: return launch_ctc_grad<4, 8>(alpha, log_probs, targets, in_lens, tgt_lens, grad_loss, z, p, B, T, V, S, grad, st);
        case 88: return launch_ctc_grad<8, 8>(alpha, log_probs, targets, in_lens, tgt_lens, grad_loss, z, p, B, T, V, S, grad, st);
        case 168: return launch_ctc_grad<16, 8>(alpha, log_probs, targets, in_lens, tgt_lens, grad_loss, z, p, B, T, V, S, grad, st);
        case 1616: return launch_ctc_grad<16, 16>(alpha, log_probs, targets, in_lens, tgt_lens, grad_loss, z, p, B, T, V, S, grad, st);
        default: return ASR_ERR_UNSUPPORTED;
    }
}

}  // namespace asr

extern "C" int asr_ctc_grad(const double* alpha, const float* log_Z, const float* log_probs, const int32_t* targets,
                            const int32_t* in_lens, const int32_t* tgt_lens, const float* grad_loss,
                            int zero_infinity, int B, int T, int V, int S, float* grad_logits, asr_stream_t stream) {
    NvtxRange range("asr::ctc_grad");
    if (B < 0 || T < 1 || V < 1 || S < 0) return ASR_ERR_INVALID_ARGUMENT;
    if (B == 0) return ASR_OK;
    if (!alpha || !log_Z || !log_probs || !in_lens || !tgt_lens || !grad_loss || !grad_logits ||
        (S > 0 && !targets))
        return ASR_ERR_INVALID_ARGUMENT;
    return ctc_grad_dispatch(alpha, log_probs, targets, in_lens, tgt_lens, grad_loss, zero_infinity, 0, B, T, V, S,
                             grad_logits, reinterpret_cast<cudaStream_t>(stream));
}
