// Fused CTC head: RMSNorm + Linear + log-softmax + CTC loss, forward and
// backward, without the (B, T, V) logits or log-probs in HBM.
//
// The reference CTC system (src/asr/system/ctc.py:21-24, :36-40) evaluates
//   logits = Linear(RMSNorm(enc))        (autocast: bf16 GEMM, fp32 accumulation)
//   loss   = CTCLoss(logits)             (log_softmax in fp32 + the CTC DP,
//                                         src/asr/loss/ctc.py:11-30)
// and its backward writes d loss / d logits for all V columns before two more
// GEMMs. Here a CTC frame is a transducer lattice node with one label position
// (U_b = 1), so the tensor-core joint (joint_tc.cu, head mode) runs the vocabulary
// GEMM with the RMSNorm rows and the bias as a ones column:
//   forward : lattice_prep -> slot_prep (unique labels of each utterance) ->
//             joint forward (per-frame log-partition + blank log-prob) ->
//             label logits (per-utterance GEMM against the K_b label rows only) ->
//             CTC alpha over the compact (B, T, K) emission table, K = S + 1
//             slots (slot 0 = blank; targets rewritten as slot ids, so the
//             recursion of ctc.cu runs unchanged)
//   backward: CTC beta -> grad_loss x slot posteriors (B, T, K) ->
//             joint backward with G = grad_loss * softmax (dense part; its dH
//             epilogue writes d hidden rows, its dW epilogue also the bias
//             gradient) -> sparse part (the posterior terms, K_b labels per
//             utterance) -> RMSNorm backward.
#include <algorithm>
#include <cstring>

#include "joint.cuh"

namespace asr {
namespace {

constexpr int kHeadThreads = 256;
constexpr int kFrameTile = 32;   // frames per tile
constexpr int kLabelBlock = 128; // label slots per block
constexpr int kColChunk = 128;   // hidden columns per chunk

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

template <typename TA>
__device__ __forceinline__ float ld_act(const TA* p) {
    if constexpr (sizeof(TA) == 2)
        return __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(p));
    else
        return __ldg(reinterpret_cast<const float*>(p));
}

// Unique labels of each utterance in first-occurrence order: slot 0 is the blank
// (vocabulary id 0), slots 1..K_b-1 the distinct target labels; slot_tg maps each
// target position to its slot. Labels outside [0, V) are clamped into it so no
// weight-row access leaves the matrix (the reference leaves them undefined). One
// warp per utterance: the lanes compare a label against 32 known slots at a time
// in shared memory.
constexpr int kSlotWarps = 4;

__global__ void __launch_bounds__(32 * kSlotWarps) slot_prep_kernel(const int32_t* __restrict__ targets,
                                                                    const int32_t* __restrict__ tgt_lens, int B,
                                                                    int S, int K, int V, int32_t* __restrict__ labels,
                                                                    int32_t* __restrict__ kb,
                                                                    int32_t* __restrict__ slot_tg) {
    extern __shared__ int32_t slot_smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int b = blockIdx.x * kSlotWarps + warp;
    if (b >= B) return;
    int32_t* L = slot_smem + warp * K;
    const int Sb = min(max(tgt_lens[b], 0), S);
    int n = 1;
    if (lane == 0) L[0] = 0;
    __syncwarp();
    for (int s = 0; s < S; ++s) {
        int slot = 0;
        if (s < Sb) {
            const int y = min(max(targets[(int64_t)b * S + s], 0), V - 1);
            slot = -1;
            for (int j0 = 0; j0 < n && slot < 0; j0 += 32) {
                const int j = j0 + lane;
                const unsigned hit = __ballot_sync(0xffffffffu, j < n && L[j] == y);
                if (hit) slot = j0 + __ffs(hit) - 1;
            }
            if (slot < 0) {
                slot = n;
                if (lane == 0) L[n] = y;
                ++n;
            }
            __syncwarp();
        }
        if (lane == 0) slot_tg[(int64_t)b * S + s] = slot;
    }
    for (int j = lane; j < K; j += 32) labels[(int64_t)b * K + j] = j < n ? L[j] : 0;
    if (lane == 0) kb[b] = n;
}

// rstd of the frames [t0, t0 + nf) of utterance b into rs[] (one warp per frame).
template <typename TA>
__device__ void frame_rstd(const TA* __restrict__ enc, int b, int T, int d, int t0, int nf, float eps, float* rs) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int f = warp; f < nf; f += kHeadThreads / 32) {
        const TA* x = enc + ((int64_t)b * T + t0 + f) * d;
        float ss = 0.f;
        for (int k = lane; k < d; k += 32) {
            const float v = ld_act(x + k);
            ss = fmaf(v, v, ss);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) rs[f] = rsqrtf(ss / (float)d + eps);
    }
}

// E[b, t, k] = log-prob of label slot k at frame t: slot 0 from the joint
// epilogue's blank log-prob, slots >= 1 from bf16(h) . bf16(W[label]) + bf16(bias)
// - lse (the operands the tensor-core GEMM uses). Grid (frame tiles, B).
template <typename TA>
__global__ void __launch_bounds__(kHeadThreads) label_logits_kernel(
    LatticeMeta m, const TA* __restrict__ enc, const float* __restrict__ g, float eps, const float* __restrict__ W,
    const float* __restrict__ bias, const int32_t* __restrict__ labels, const int32_t* __restrict__ kb,
    const float* __restrict__ lse, const float* __restrict__ lpb, int T, int d, int K, float* __restrict__ E) {
    extern __shared__ float head_smem[];
    auto hs = reinterpret_cast<float(*)[kColChunk + 1]>(head_smem);                               // [kFrameTile]
    auto ws = reinterpret_cast<float(*)[kColChunk + 1]>(head_smem + kFrameTile * (kColChunk + 1));  // [kLabelBlock]
    __shared__ float rs[kFrameTile];
    const int b = blockIdx.y, t0 = blockIdx.x * kFrameTile;
    const int Tb = __ldg(m.Tb + b);
    if (t0 >= Tb) return;
    const int nf = min(kFrameTile, Tb - t0), Kb = __ldg(kb + b), off = __ldg(m.off + b);
    const int32_t* L = labels + (int64_t)b * K;
    frame_rstd(enc, b, T, d, t0, nf, eps, rs);
    // thread tile: frames fg*4 .. +3 x labels lg*4 .. +3 (8 frame groups x 32 label groups)
    const int fg = threadIdx.x % 8, lg = threadIdx.x / 8;
    for (int l0 = 0; l0 < Kb; l0 += kLabelBlock) {
        float acc[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int q = 0; q < 4; ++q) acc[i][q] = 0.f;
        for (int k0 = 0; k0 < d; k0 += kColChunk) {
            __syncthreads();  // rs ready / previous chunk consumed
            for (int i = threadIdx.x; i < kFrameTile * kColChunk; i += kHeadThreads) {
                const int ff = i / kColChunk, kk = i % kColChunk, k = k0 + kk;
                float h = 0.f;
                if (ff < nf && k < d) h = bf16r(ld_act(enc + ((int64_t)b * T + t0 + ff) * d + k) * rs[ff] * __ldg(g + k));
                hs[ff][kk] = h;
            }
            for (int i = threadIdx.x; i < kLabelBlock * kColChunk; i += kHeadThreads) {
                const int l = i / kColChunk, kk = i % kColChunk, k = k0 + kk;
                float w = 0.f;
                if (l0 + l < Kb && k < d) w = bf16r(__ldg(W + (int64_t)__ldg(L + l0 + l) * d + k));
                ws[l][kk] = w;
            }
            __syncthreads();
            const int kn = min(kColChunk, d - k0);
            for (int kk = 0; kk < kn; ++kk) {
                float h[4], w[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) h[i] = hs[fg * 4 + i][kk];
#pragma unroll
                for (int q = 0; q < 4; ++q) w[q] = ws[lg * 4 + q][kk];
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int q = 0; q < 4; ++q) acc[i][q] = fmaf(h[i], w[q], acc[i][q]);
            }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int f = fg * 4 + i;
            if (f >= nf) break;
            const int n = off + t0 + f;
            const float l_n = __ldg(lse + n);
            float* e = E + ((int64_t)b * T + t0 + f) * K;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int slot = l0 + lg * 4 + q;
                if (slot >= Kb) break;
                if (slot == 0) {
                    e[0] = __ldg(lpb + n);
                } else {
                    const float bb = bias ? bf16r(__ldg(bias + __ldg(L + slot))) : 0.f;
                    e[slot] = acc[i][q] + bb - l_n;
                }
            }
        }
    }
}

// Dense-part scale per frame node: G = cb * softmax (zero for utterances whose
// loss zero_infinity drops).
__global__ void fill_cb_kernel(LatticeMeta m, int B, const float* __restrict__ grad_loss,
                               const float* __restrict__ logz, int zero_infinity, float* __restrict__ cb,
                               float* __restrict__ ct) {
    const int N = total_nodes(m, B);
    for (int n = blockIdx.x * blockDim.x + threadIdx.x; n < N; n += gridDim.x * blockDim.x) {
        const int b = find_utt(m.off, B, n);
        const bool dead = zero_infinity && !isfinite(__ldg(logz + b));
        cb[n] = dead ? 0.f : __ldg(grad_loss + b);
        ct[n] = 0.f;
    }
}

// Sparse part of the backward: with P[b, t, k] = grad_loss * posterior of slot k,
//   d_hidden[b, t, :] -= sum_k P[t, k] W[label_k]      (RMW: this CTA owns the column chunk)
//   dW[label_k, :]    -= sum_t P[t, k] h[t]            (one atomic per element per CTA)
//   d_bias[label_k]   -= sum_t P[t, k]                 (column chunk 0)
// Grid (column chunks, B); each CTA walks all frames of its utterance.
template <typename TA>
__global__ void __launch_bounds__(kHeadThreads) sparse_bwd_kernel(
    LatticeMeta m, const TA* __restrict__ enc, const float* __restrict__ g, float eps, const float* __restrict__ W,
    const int32_t* __restrict__ labels, const int32_t* __restrict__ kb, const float* __restrict__ P, int T, int d,
    int K, float* __restrict__ dh, float* __restrict__ dW, float* __restrict__ dbias) {
    extern __shared__ float head_smem[];
    auto hs = reinterpret_cast<float(*)[kColChunk + 1]>(head_smem);                               // [kFrameTile]
    auto ws = reinterpret_cast<float(*)[kColChunk + 1]>(head_smem + kFrameTile * (kColChunk + 1));  // [kLabelBlock]
    auto ps = reinterpret_cast<float(*)[kLabelBlock + 1]>(head_smem + (kFrameTile + kLabelBlock) * (kColChunk + 1));
    __shared__ float rs[kFrameTile];
    const int b = blockIdx.y, k0 = blockIdx.x * kColChunk;
    const int Tb = __ldg(m.Tb + b), Kb = __ldg(kb + b);
    const int32_t* L = labels + (int64_t)b * K;
    // d hidden tile: frames dfg*4 .. +3 x columns dcg + 32q (q < 4)
    const int dcg = threadIdx.x % 32, dfg = threadIdx.x / 32;
    // dW tile: labels wlg*8 .. +7 x columns wcg + 16q (q < 8)
    const int wcg = threadIdx.x % 16, wlg = threadIdx.x / 16;
    for (int l0 = 0; l0 < Kb; l0 += kLabelBlock) {
        const int nl = min(kLabelBlock, Kb - l0);
        __syncthreads();
        for (int i = threadIdx.x; i < kLabelBlock * kColChunk; i += kHeadThreads) {
            const int l = i / kColChunk, c = i % kColChunk;
            float w = 0.f;
            if (l < nl && k0 + c < d) w = bf16r(__ldg(W + (int64_t)__ldg(L + l0 + l) * d + k0 + c));
            ws[l][c] = w;
        }
        float dwacc[8][8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int q = 0; q < 8; ++q) dwacc[i][q] = 0.f;
        float dbacc = 0.f;  // thread l < nl of chunk 0: sum over frames of P[., l]
        for (int t0 = 0; t0 < Tb; t0 += kFrameTile) {
            const int nf = min(kFrameTile, Tb - t0);
            __syncthreads();
            frame_rstd(enc, b, T, d, t0, nf, eps, rs);
            for (int i = threadIdx.x; i < kFrameTile * kLabelBlock; i += kHeadThreads) {
                const int ff = i / kLabelBlock, l = i % kLabelBlock;
                ps[ff][l] = (ff < nf && l < nl) ? __ldg(P + ((int64_t)b * T + t0 + ff) * K + l0 + l) : 0.f;
            }
            __syncthreads();
            for (int i = threadIdx.x; i < kFrameTile * kColChunk; i += kHeadThreads) {
                const int ff = i / kColChunk, c = i % kColChunk;
                float h = 0.f;
                if (ff < nf && k0 + c < d)
                    h = bf16r(ld_act(enc + ((int64_t)b * T + t0 + ff) * d + k0 + c) * rs[ff] * __ldg(g + k0 + c));
                hs[ff][c] = h;
            }
            __syncthreads();
            // d hidden -= P W_labels
            {
                float acc[4][4];
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int q = 0; q < 4; ++q) acc[i][q] = 0.f;
                for (int l = 0; l < nl; ++l) {
                    float pv[4], wv[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) pv[i] = ps[dfg * 4 + i][l];
#pragma unroll
                    for (int q = 0; q < 4; ++q) wv[q] = ws[l][dcg + 32 * q];
#pragma unroll
                    for (int i = 0; i < 4; ++i)
#pragma unroll
                        for (int q = 0; q < 4; ++q) acc[i][q] = fmaf(pv[i], wv[q], acc[i][q]);
                }
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int ff = dfg * 4 + i;
                    if (ff >= nf) break;
                    float* row = dh + ((int64_t)b * T + t0 + ff) * d + k0;
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                        if (k0 + dcg + 32 * q < d) row[dcg + 32 * q] -= acc[i][q];
                }
            }
            // dW: labels x columns, summed over the frames of the tile
            for (int ff = 0; ff < nf; ++ff) {
                float pv[8], hv[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) pv[i] = ps[ff][wlg * 8 + i];
#pragma unroll
                for (int q = 0; q < 8; ++q) hv[q] = hs[ff][wcg + 16 * q];
#pragma unroll
                for (int i = 0; i < 8; ++i)
#pragma unroll
                    for (int q = 0; q < 8; ++q) dwacc[i][q] = fmaf(pv[i], hv[q], dwacc[i][q]);
            }
            if (blockIdx.x == 0 && threadIdx.x < nl)
                for (int ff = 0; ff < nf; ++ff) dbacc += ps[ff][threadIdx.x];
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int l = wlg * 8 + i;
            if (l >= nl) break;
            float* dst = dW + (int64_t)__ldg(L + l0 + l) * d + k0;
#pragma unroll
            for (int q = 0; q < 8; ++q)
                if (k0 + wcg + 16 * q < d) atomicAdd(dst + wcg + 16 * q, -dwacc[i][q]);
        }
        if (dbias && blockIdx.x == 0 && threadIdx.x < nl) atomicAdd(dbias + __ldg(L + l0 + threadIdx.x), -dbacc);
    }
}

// RMSNorm backward over every (b, t) row: with x^ = x * rstd and dy = d hidden,
//   d_x = rstd * (g * dy - x^ * mean(x^ * g * dy)),   d_g += dy * x^,
// zero rows past in_lens[b]. 32 rows per CTA; d_g summed per CTA, one atomic per
// column.
template <typename TA>
__global__ void __launch_bounds__(kHeadThreads) rms_bwd_kernel(LatticeMeta m, const TA* __restrict__ enc,
                                                               const float* __restrict__ g, float eps,
                                                               const float* __restrict__ dh, int B, int T, int d,
                                                               TA* __restrict__ d_enc, float* __restrict__ dg) {
    __shared__ float rs[kFrameTile], cs[kFrameTile];
    __shared__ int live[kFrameTile];
    const int64_t row0 = (int64_t)blockIdx.x * kFrameTile;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int f = warp; f < kFrameTile; f += kHeadThreads / 32) {
        const int64_t r = row0 + f;
        int ok = 0;
        float rstd = 0.f, c = 0.f;
        if (r < (int64_t)B * T) {
            const int b = (int)(r / T), t = (int)(r % T);
            ok = t < __ldg(m.Tb + b);
        }
        if (ok) {
            const TA* x = enc + r * d;
            const float* dy = dh + r * d;
            float ss = 0.f, sd = 0.f;
            for (int k = lane; k < d; k += 32) {
                const float v = ld_act(x + k);
                ss = fmaf(v, v, ss);
                sd = fmaf(v * __ldg(g + k), dy[k], sd);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                ss += __shfl_xor_sync(0xffffffffu, ss, o);
                sd += __shfl_xor_sync(0xffffffffu, sd, o);
            }
            rstd = rsqrtf(ss / (float)d + eps);
            c = sd * rstd / (float)d;  // mean(x^ * g * dy)
        }
        if (lane == 0) {
            rs[f] = rstd;
            cs[f] = c;
            live[f] = ok;
        }
    }
    __syncthreads();
    for (int k = threadIdx.x; k < d; k += kHeadThreads) {
        const float gk = __ldg(g + k);
        float acc = 0.f;
        for (int f = 0; f < kFrameTile; ++f) {
            const int64_t r = row0 + f;
            if (r >= (int64_t)B * T) break;
            float dx = 0.f;
            if (live[f]) {
                const float xh = ld_act(enc + r * d + k) * rs[f];
                const float dy = dh[r * d + k];
                dx = rs[f] * (gk * dy - xh * cs[f]);
                acc = fmaf(dy, xh, acc);
            }
            if constexpr (sizeof(TA) == 2)
                reinterpret_cast<__nv_bfloat16*>(d_enc)[r * d + k] = __float2bfloat16_rn(dx);
            else
                reinterpret_cast<float*>(d_enc)[r * d + k] = dx;
        }
        atomicAdd(dg + k, acc);
    }
}

__global__ void head_loss_kernel(const float* __restrict__ logz, int B, int zero_infinity, float* __restrict__ loss) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    const float l = -logz[b];
    loss[b] = (zero_infinity && !isfinite(l)) ? 0.f : l;
}

size_t al256(size_t x) { return (x + 255) & ~size_t(255); }

constexpr size_t kLogitSmem = sizeof(float) * (kFrameTile + kLabelBlock) * (kColChunk + 1);
constexpr size_t kSparseSmem = kLogitSmem + sizeof(float) * kFrameTile * (kLabelBlock + 1);

// One workspace serves a forward and the backward of the same call: the forward
// leaves the per-frame log-partition, the emission table and alpha in it.
struct HeadWs {
    LatticeMeta meta;
    int32_t *labels, *kb, *slot_tg;
    float *lse, *lpb, *lpy, *E, *logz, *P, *cb, *ct, *dh;
    double* alpha;
    void* joint;
    size_t joint_bytes, total;
};

JointArgs head_args(const void* enc, int act_dtype, const float* rms_g, float eps, const float* W,
                    const float* bias, int B, int T, int V, int d) {
    JointArgs a;
    std::memset(&a, 0, sizeof(a));
    if (act_dtype == ASR_DTYPE_BF16)
        a.enc16 = static_cast<const __nv_bfloat16*>(enc);
    else
        a.enc = static_cast<const float*>(enc);
    a.W = W;
    a.B = B;
    a.T = T;
    a.U = 1;
    a.V = V;
    a.d = d;
    a.S = 0;
    a.blank = 0;
    a.head = 1;
    a.rms_g = rms_g;
    a.rms_eps = eps;
    a.bias = bias;
    return a;
}

HeadWs head_layout(void* base, const JointArgs& a, int S) {
    HeadWs w;
    std::memset(&w, 0, sizeof(w));
    const int B = a.B, T = a.T, K = S + 1;
    const int64_t cap = (int64_t)B * T;
    char* p0 = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(base) + 255) & ~uintptr_t(255));
    char* p = p0;
    if (base) p = lattice_meta_carve(p, B, &w.meta);
    else p += lattice_meta_bytes(B);
    auto take = [&](size_t bytes) {
        char* o = p;
        p += al256(bytes);
        return o;
    };
    w.labels = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * B * K));
    w.kb = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * B));
    w.slot_tg = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * B * std::max(S, 1)));
    w.lse = reinterpret_cast<float*>(take(sizeof(float) * cap));
    w.lpb = reinterpret_cast<float*>(take(sizeof(float) * cap));
    w.lpy = reinterpret_cast<float*>(take(sizeof(float) * cap));
    w.E = reinterpret_cast<float*>(take(sizeof(float) * cap * K));
    w.logz = reinterpret_cast<float*>(take(sizeof(float) * B));
    w.alpha = reinterpret_cast<double*>(take(sizeof(double) * cap * (2 * S + 1)));
    w.P = reinterpret_cast<float*>(take(sizeof(float) * cap * K));
    w.cb = reinterpret_cast<float*>(take(sizeof(float) * cap));
    w.ct = reinterpret_cast<float*>(take(sizeof(float) * cap));
    w.dh = reinterpret_cast<float*>(take(sizeof(float) * cap * a.d));
    w.joint_bytes = std::max(tc_forward_scratch_bytes(a, (int)cap), tc_backward_scratch_bytes(a, (int)cap));
    w.joint = take(w.joint_bytes);
    w.total = (size_t)(p - p0) + 256;
    return w;
}

bool head_bad(int B, int T, int S, int V, int d, int act_dtype) {
    return B < 0 || T < 1 || S < 0 || V < 1 || d < 1 || (act_dtype != ASR_DTYPE_F32 && act_dtype != ASR_DTYPE_BF16);
}

template <typename TA>
int head_forward(const JointArgs& a, const HeadWs& w, const TA* enc, const int32_t* targets,
                 const int32_t* in_lens, const int32_t* tgt_lens, int S, int zero_infinity, float* loss,
                 cudaStream_t st) {
    const int B = a.B, T = a.T, K = S + 1;
    const int64_t cap = (int64_t)B * T;
    int rc = launch_lattice_prep(in_lens, tgt_lens, B, T, 1, S, w.meta, st);
    if (rc) return rc;
    {
        KernelTimer kt("ctc_head_slots", st);
        const size_t smem = sizeof(int32_t) * (size_t)K * kSlotWarps;
        ASR_CUDA_TRY(cudaFuncSetAttribute(slot_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        slot_prep_kernel<<<(B + kSlotWarps - 1) / kSlotWarps, 32 * kSlotWarps, smem, st>>>(
            targets, tgt_lens, B, S, K, a.V, w.labels, w.kb, w.slot_tg);
        ASR_LAUNCH_CHECK();
    }
    JointFwdOut o{w.lpb, w.lse, w.lpy, nullptr};
    rc = tc_joint_forward(a, o, (int)cap, w.joint, w.joint_bytes, st);
    if (rc) return rc;
    {
        KernelTimer kt("ctc_head_label_logits", st);
        const dim3 grid((T + kFrameTile - 1) / kFrameTile, B);
        ASR_CUDA_TRY(cudaFuncSetAttribute(label_logits_kernel<TA>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)kLogitSmem));
        label_logits_kernel<TA><<<grid, kHeadThreads, kLogitSmem, st>>>(w.meta, enc, a.rms_g, a.rms_eps, a.W, a.bias,
                                                                w.labels, w.kb, w.lse, w.lpb, T, a.d, K, w.E);
        ASR_LAUNCH_CHECK();
    }
    double* alpha = w.alpha;
    rc = asr_ctc_alpha(w.E, w.slot_tg, in_lens, tgt_lens, B, T, K, S, alpha, w.logz,
                       reinterpret_cast<asr_stream_t>(st));
    if (rc) return rc;
    head_loss_kernel<<<(B + 127) / 128, 128, 0, st>>>(w.logz, B, zero_infinity, loss);
    ASR_LAUNCH_CHECK();
    return ASR_OK;
}

template <typename TA>
int head_backward(const JointArgs& a, const HeadWs& w, const TA* enc, const int32_t* in_lens,
                  const int32_t* tgt_lens, int S, int zero_infinity, const float* grad_loss, TA* grad_enc,
                  float* grad_g, float* grad_W, float* grad_bias, cudaStream_t st) {
    const int B = a.B, T = a.T, K = S + 1;
    const int64_t cap = (int64_t)B * T;
    int rc = launch_lattice_prep(in_lens, tgt_lens, B, T, 1, S, w.meta, st);
    if (rc) return rc;
    rc = ctc_grad_dispatch(w.alpha, w.E, w.slot_tg, in_lens, tgt_lens, grad_loss, zero_infinity, 1, B, T, K, S, w.P,
                           st);
    if (rc) return rc;
    {
        KernelTimer kt("ctc_head_prep_bwd", st);
        fill_cb_kernel<<<sm_count() * 4, 256, 0, st>>>(w.meta, B, grad_loss, w.logz, zero_infinity, w.cb, w.ct);
        ASR_LAUNCH_CHECK();
    }
    ASR_CUDA_TRY(cudaMemsetAsync(w.dh, 0, sizeof(float) * cap * a.d, st));
    ASR_CUDA_TRY(cudaMemsetAsync(grad_W, 0, sizeof(float) * (size_t)a.V * a.d, st));
    ASR_CUDA_TRY(cudaMemsetAsync(grad_g, 0, sizeof(float) * (size_t)a.d, st));
    if (grad_bias) ASR_CUDA_TRY(cudaMemsetAsync(grad_bias, 0, sizeof(float) * (size_t)a.V, st));
    JointArgs ab = a;
    ab.blank = -1;  // G = cb * softmax: no blank term in the dense part
    JointBwdIn in{w.lse, w.cb, w.ct, nullptr};
    JointBwdOut o{w.dh, nullptr, grad_W, nullptr, grad_bias};
    rc = tc_joint_backward(ab, in, o, (int)cap, w.joint, w.joint_bytes, st);
    if (rc) return rc;
    {
        KernelTimer kt("ctc_head_sparse_bwd", st);
        const dim3 grid((a.d + kColChunk - 1) / kColChunk, B);
        ASR_CUDA_TRY(cudaFuncSetAttribute(sparse_bwd_kernel<TA>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)kSparseSmem));
        sparse_bwd_kernel<TA><<<grid, kHeadThreads, kSparseSmem, st>>>(w.meta, enc, a.rms_g, a.rms_eps, a.W, w.labels, w.kb,
                                                              w.P, T, a.d, K, w.dh, grad_W, grad_bias);
        ASR_LAUNCH_CHECK();
    }
    {
        KernelTimer kt("ctc_head_rms_bwd", st);
        rms_bwd_kernel<TA><<<(unsigned)((cap + kFrameTile - 1) / kFrameTile), kHeadThreads, 0, st>>>(
            w.meta, enc, a.rms_g, a.rms_eps, w.dh, B, T, a.d, grad_enc, grad_g);
        ASR_LAUNCH_CHECK();
    }
    return ASR_OK;
}

}  // namespace
}  // namespace asr

using namespace asr;

extern "C" size_t asr_ctc_head_workspace_bytes(int B, int T, int S, int V, int d, int act_dtype) {
    if (head_bad(B, T, S, V, d, act_dtype) || B == 0) return 0;
    JointArgs a = head_args(nullptr, act_dtype, nullptr, 0.f, nullptr, reinterpret_cast<const float*>(16), B, T, V, d);
    return head_layout(nullptr, a, S).total;
}

extern "C" int asr_ctc_head_supported(int V, int d) {
    JointArgs a = head_args(nullptr, ASR_DTYPE_F32, nullptr, 0.f, nullptr, reinterpret_cast<const float*>(16), 1, 1,
                            V, d);
    return tc_backward_supported(a) ? 1 : 0;
}

extern "C" int asr_ctc_head_forward(const void* encoder, int act_dtype, const float* rms_weight, float rms_eps,
                                    const float* weight, const float* bias, const int32_t* targets,
                                    const int32_t* in_lens, const int32_t* tgt_lens, int B, int T, int S, int V, int d,
                                    int zero_infinity, float* loss, void* workspace, size_t workspace_bytes,
                                    asr_stream_t stream) {
    if (head_bad(B, T, S, V, d, act_dtype)) return ASR_ERR_INVALID_ARGUMENT;
    if (B == 0) return ASR_OK;
    if (!encoder || !rms_weight || !weight || !in_lens || !tgt_lens || !loss || (S > 0 && !targets))
        return ASR_ERR_INVALID_ARGUMENT;
    if (2 * S + 1 > 1024) return ASR_ERR_UNSUPPORTED;
    JointArgs a = head_args(encoder, act_dtype, rms_weight, rms_eps, weight, bias, B, T, V, d);
    if (!tc_backward_supported(a)) return ASR_ERR_UNSUPPORTED;
    HeadWs w = head_layout(workspace, a, S);
    if (!workspace || workspace_bytes < w.total) return ASR_ERR_WORKSPACE;
    a.m = w.meta;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (act_dtype == ASR_DTYPE_BF16)
        return head_forward(a, w, static_cast<const __nv_bfloat16*>(encoder), targets, in_lens, tgt_lens, S,
                            zero_infinity, loss, st);
    return head_forward(a, w, static_cast<const float*>(encoder), targets, in_lens, tgt_lens, S, zero_infinity, loss,
                        st);
}

extern "C" int asr_ctc_head_backward(const void* encoder, int act_dtype, const float* rms_weight, float rms_eps,
                                     const float* weight, const float* bias, const int32_t* targets,
                                     const int32_t* in_lens, const int32_t* tgt_lens, int B, int T, int S, int V,
                                     int d, int zero_infinity, const float* grad_loss, void* grad_encoder,
                                     float* grad_rms_weight, float* grad_weight, float* grad_bias, void* workspace,
                                     size_t workspace_bytes, asr_stream_t stream) {
    if (head_bad(B, T, S, V, d, act_dtype)) return ASR_ERR_INVALID_ARGUMENT;
    if (!grad_rms_weight || !grad_weight || (bias && !grad_bias)) return ASR_ERR_INVALID_ARGUMENT;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (B == 0) {
        ASR_CUDA_TRY(cudaMemsetAsync(grad_weight, 0, sizeof(float) * (size_t)V * d, st));
        ASR_CUDA_TRY(cudaMemsetAsync(grad_rms_weight, 0, sizeof(float) * (size_t)d, st));
        if (grad_bias) ASR_CUDA_TRY(cudaMemsetAsync(grad_bias, 0, sizeof(float) * (size_t)V, st));
        return ASR_OK;
    }
    if (!encoder || !rms_weight || !weight || !in_lens || !tgt_lens || !grad_loss || !grad_encoder ||
        (S > 0 && !targets))
        return ASR_ERR_INVALID_ARGUMENT;
    (void)targets;  // the forward left the slot tables in the workspace
    if (2 * S + 1 > 1024) return ASR_ERR_UNSUPPORTED;
    JointArgs a = head_args(encoder, act_dtype, rms_weight, rms_eps, weight, bias, B, T, V, d);
    if (!tc_backward_supported(a)) return ASR_ERR_UNSUPPORTED;
    HeadWs w = head_layout(workspace, a, S);
    if (!workspace || workspace_bytes < w.total) return ASR_ERR_WORKSPACE;
    a.m = w.meta;
    if (act_dtype == ASR_DTYPE_BF16)
        return head_backward(a, w, static_cast<const __nv_bfloat16*>(encoder), in_lens, tgt_lens, S, zero_infinity,
                             grad_loss, static_cast<__nv_bfloat16*>(grad_encoder), grad_rms_weight, grad_weight,
                             grad_bias, st);
    return head_backward(a, w, static_cast<const float*>(encoder), in_lens, tgt_lens, S, zero_infinity, grad_loss,
                         static_cast<float*>(grad_encoder), grad_rms_weight, grad_weight, grad_bias, st);
}
