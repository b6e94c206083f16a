// TDT lattice recursions on the (T_b + 1)-frame grid: alpha (forward) and beta
// fused with the edge posteriors and the duration-head logit gradient
// (backward). Reference semantics: tdt.cu:195-428, tests/loss/tdt_reference.py:109-356.
//
// Every TDT edge leaves node (t, u) on anti-diagonal g = t + u and lands on a
// strictly later diagonal: a blank of duration d lands on g + d (d >= 1) and a
// token of duration d lands on g + d + 1 (d >= 0, so the intra-frame d = 0 chain
// is just a distance-1 edge). One warp sweeps the diagonals of one utterance,
// lane l owning label positions u = l*K .. l*K+K-1 in registers:
//  * forward (push): when node (t, u) is final it adds alpha + edge weight into
//    a register ring of the next MAXD+1 diagonals (blank: same register, token:
//    the next register, or the next lane's head register via one shuffle per
//    duration);
//  * backward (pull): beta(t, u) reads a ring of the previous MAXD+1 diagonals
//    of its own register and of the next label position, then the same values
//    give every edge posterior of (t, u) in place.
// Durations are arbitrary (duplicates allowed): for each duration value the
// matching duration classes are kept as a bit mask and their log-probs are
// log-summed. As in the reference, the d = 0 token chain of the recursions uses
// the first zero-duration class only, while posteriors cover every class.
#include "dp.cuh"

namespace asr {
namespace {

constexpr int kDpWarps = 4;

__device__ __forceinline__ float lse_mask(const float* __restrict__ ld, uint32_t mask) {
    float w = kNeg;
    bool first = true;
    while (mask) {
        const int k = __ffs(mask) - 1;
        mask &= mask - 1;
        const float x = ld[k];
        w = first ? x : lae(w, x);
        first = false;
    }
    return w;
}

template <int MAXD>
__device__ __forceinline__ void duration_masks(const int32_t* __restrict__ durations, int n_dur, int has_zero,
                                               uint32_t (&dmask)[MAXD + 1], uint32_t& tok0) {
#pragma unroll
    for (int dv = 0; dv <= MAXD; ++dv) dmask[dv] = 0u;
    int zk = -1;
    for (int k = 0; k < n_dur; ++k) {
        const int dk = durations[k];
#pragma unroll
        for (int dv = 0; dv <= MAXD; ++dv)
            if (dk == dv) dmask[dv] |= 1u << k;
        if (dk == 0 && zk < 0) zk = k;
    }
    tok0 = (has_zero && zk >= 0) ? (1u << zk) : 0u;
}

template <int K, int MAXD>
__global__ void __launch_bounds__(32 * kDpWarps)
    tdt_alpha_kernel(LatticeMeta m, int B, const int32_t* __restrict__ durations, int n_dur, int has_zero,
                     const float* __restrict__ lpb, const float* __restrict__ lpy, const float* __restrict__ lpd,
                     double* __restrict__ alpha, float* __restrict__ log_prob, float* __restrict__ loss) {
    constexpr int R = MAXD + 2;  // slot r accumulates edges landing on diagonal g + r
    const int lane = threadIdx.x & 31;
    const int b = blockIdx.x * kDpWarps + (threadIdx.x >> 5);
    if (b >= B) return;
    uint32_t dmask[MAXD + 1], tok0;
    duration_masks<MAXD>(durations, n_dur, has_zero, dmask, tok0);
    const int Tb = m.Tb[b], Ub = m.Ub[b], off = m.off[b], aoff = m.aoff[b];

    double acc[K][R];
#pragma unroll
    for (int j = 0; j < K; ++j)
#pragma unroll
        for (int r = 0; r < R; ++r) acc[j][r] = kNeg;
    if (lane == 0) acc[0][0] = 0.0;  // start node (0, 0)

    const int last = Tb + Ub - 1;
    for (int g = 0; g <= last; ++g) {
        double tokout[MAXD + 1];
#pragma unroll
        for (int dv = 0; dv <= MAXD; ++dv) tokout[dv] = kNeg;
        double a[K];
#pragma unroll
        for (int j = 0; j < K; ++j) a[j] = acc[j][0];
#pragma unroll
        for (int j = 0; j < K; ++j) {
            const int u = lane * K + j, t = g - u;
            if (u < Ub && t >= 0 && t <= Tb) {
                alpha[aoff + t * Ub + u] = a[j];
                if (t == Tb && u == Ub - 1) {  // exact-landing terminal (tdt.cu:291-295)
                    log_prob[b] = (float)a[j];
                    loss[b] = (float)(-a[j]);
                }
                if (t < Tb) {
                    const int n = off + t * Ub + u;
                    const float lb = lpb[n], ly = lpy[n];
                    const float* ld = lpd + (int64_t)n * n_dur;
#pragma unroll
                    for (int dv = 1; dv <= MAXD; ++dv) {
                        if (dmask[dv] && t + dv <= Tb)
                            acc[j][dv] = lae_d(acc[j][dv], a[j] + lb + lse_mask(ld, dmask[dv]));
                    }
                    if (u < Ub - 1) {
#pragma unroll
                        for (int dv = 0; dv <= MAXD; ++dv) {
                            const uint32_t mk = dv == 0 ? tok0 : dmask[dv];
                            if (mk && t + dv <= Tb) {
                                const double v = a[j] + ly + lse_mask(ld, mk);
                                if (j + 1 < K)
                                    acc[(j + 1) % K][dv + 1] = lae_d(acc[(j + 1) % K][dv + 1], v);
                                else
                                    tokout[dv] = v;
                            }
                        }
                    }
                }
            }
        }
#pragma unroll
        for (int dv = 0; dv <= MAXD; ++dv) {
            const double x = __shfl_up_sync(0xffffffffu, tokout[dv], 1);
            if (lane > 0 && x > kNeg) acc[0][dv + 1] = lae_d(acc[0][dv + 1], x);
        }
#pragma unroll
        for (int j = 0; j < K; ++j) {
#pragma unroll
            for (int r = 0; r + 1 < R; ++r) acc[j][r] = acc[j][r + 1];
            acc[j][R - 1] = kNeg;
        }
    }
}

// Writes per node: cb = gl * blank posterior, ct = gl * token posterior (both summed
// over durations) and gdur[k] = d loss / d duration-logit k (tdt.cu:400-426 + 475-500).
template <int K, int MAXD>
__global__ void __launch_bounds__(32 * kDpWarps)
    tdt_beta_kernel(LatticeMeta m, int B, const int32_t* __restrict__ durations, int n_dur, int has_zero,
                    const float* __restrict__ lpb, const float* __restrict__ lpy, const float* __restrict__ lpd,
                    const double* __restrict__ alpha, const float* __restrict__ grad_loss, float* __restrict__ cb,
                    float* __restrict__ ct, float* __restrict__ gdur) {
    constexpr int R = MAXD + 2;  // slot r (r >= 1) holds beta on diagonal g + r
    __shared__ float gin_all[kDpWarps][32][kTdtMaxDurClasses + 1];
    const int lane = threadIdx.x & 31;
    const int w = threadIdx.x >> 5;
    const int b = blockIdx.x * kDpWarps + w;
    if (b >= B) return;
    float* gi = gin_all[w][lane];
    uint32_t dmask[MAXD + 1], tok0;
    duration_masks<MAXD>(durations, n_dur, has_zero, dmask, tok0);
    const int Tb = m.Tb[b], Ub = m.Ub[b], off = m.off[b], aoff = m.aoff[b];
    const double logZ = alpha[aoff + Tb * Ub + Ub - 1];  // exact-landing terminal, float64
    const float gl = grad_loss[b];

    double br[K][R], nbr[R];  // own registers / next lane's head register
#pragma unroll
    for (int r = 0; r < R; ++r) {
        nbr[r] = kNeg;
#pragma unroll
        for (int j = 0; j < K; ++j) br[j][r] = kNeg;
    }
    for (int g = Tb + Ub - 1; g >= 0; --g) {
        double nbeta[K];
#pragma unroll
        for (int j = 0; j < K; ++j) {
            const int u = lane * K + j, t = g - u;
            nbeta[j] = kNeg;
            if (u < Ub && t >= 0 && t <= Tb) {
                if (t == Tb) {
                    nbeta[j] = (u == Ub - 1) ? 0.0 : (double)kNeg;  // terminal seed (tdt.cu:331,351)
                } else {
                    const int n = off + t * Ub + u;
                    const float lb = lpb[n], ly = lpy[n];
                    const double a = alpha[aoff + t * Ub + u];
                    const float* ld = lpd + (int64_t)n * n_dur;
                    const bool can_tok = u < Ub - 1;
                    double be = kNeg;
#pragma unroll
                    for (int dv = 1; dv <= MAXD; ++dv)
                        if (dmask[dv] && t + dv <= Tb) be = lae_d(be, lb + lse_mask(ld, dmask[dv]) + br[j][dv]);
                    if (can_tok) {
#pragma unroll
                        for (int dv = 0; dv <= MAXD; ++dv) {
                            const uint32_t mk = dv == 0 ? tok0 : dmask[dv];
                            const double nv = (j + 1 < K) ? br[(j + 1) % K][dv + 1] : nbr[dv + 1];
                            if (mk && t + dv <= Tb) be = lae_d(be, ly + lse_mask(ld, mk) + nv);
                        }
                    }
                    nbeta[j] = be;
                    // edge posteriors of (t, u), every duration class
                    for (int k = 0; k < n_dur; ++k) gi[k] = 0.f;
                    float bp = 0.f, tp = 0.f;
#pragma unroll
                    for (int dv = 0; dv <= MAXD; ++dv) {
                        if (t + dv > Tb) continue;
                        const double nv = (j + 1 < K) ? br[(j + 1) % K][dv + 1] : nbr[dv + 1];
                        uint32_t mk = dmask[dv];
                        while (mk) {
                            const int k = __ffs(mk) - 1;
                            mk &= mk - 1;
                            const float x = ld[k];
                            const float gbk = (dv >= 1) ? __expf((float)(a + lb + x + br[j][dv] - logZ)) : 0.f;
                            const float gtk = can_tok ? __expf((float)(a + ly + x + nv - logZ)) : 0.f;
                            bp += gbk;
                            tp += gtk;
                            gi[k] = -(gbk + gtk);
                        }
                    }
                    float gsum = 0.f;
                    for (int k = 0; k < n_dur; ++k) gsum += gi[k];
                    for (int k = 0; k < n_dur; ++k) gdur[(int64_t)n * n_dur + k] = gl * (gi[k] - __expf(ld[k]) * gsum);
                    cb[n] = gl * bp;
                    ct[n] = gl * tp;
                }
            }
        }
        double head = __shfl_down_sync(0xffffffffu, nbeta[0], 1);
        if (lane == 31) head = kNeg;
#pragma unroll
        for (int r = R - 1; r >= 2; --r) {
            nbr[r] = nbr[r - 1];
#pragma unroll
            for (int j = 0; j < K; ++j) br[j][r] = br[j][r - 1];
        }
        nbr[1] = head;
#pragma unroll
        for (int j = 0; j < K; ++j) br[j][1] = nbeta[j];
    }
}

template <int K, int MAXD>
int tdt_alpha_launch(const LatticeMeta& m, int B, const int32_t* dur, int nd, int hz, const float* lpb,
                     const float* lpy, const float* lpd, double* alpha, float* lp, float* loss, cudaStream_t st) {
    KernelTimer kt("tdt_alpha", st);
    tdt_alpha_kernel<K, MAXD><<<(B + kDpWarps - 1) / kDpWarps, 32 * kDpWarps, 0, st>>>(m, B, dur, nd, hz, lpb, lpy,
                                                                                     lpd, alpha, lp, loss);
    ASR_LAUNCH_CHECK();
    return ASR_OK;
}

template <int K, int MAXD>
int tdt_beta_launch(const LatticeMeta& m, int B, const int32_t* dur, int nd, int hz, const float* lpb,
                    const float* lpy, const float* lpd, const double* alpha, const float* gl, float* cb, float* ct,
                    float* gdur, cudaStream_t st) {
    KernelTimer kt("tdt_beta_posteriors", st);
    tdt_beta_kernel<K, MAXD><<<(B + kDpWarps - 1) / kDpWarps, 32 * kDpWarps, 0, st>>>(
        m, B, dur, nd, hz, lpb, lpy, lpd, alpha, gl, cb, ct, gdur);
    ASR_LAUNCH_CHECK();
    return ASR_OK;
}

int tdt_maxd_bucket(int max_duration) {
    if (max_duration <= 2) return 2;
    if (max_duration <= 4) return 4;
    if (max_duration <= 8) return 8;
    if (max_duration <= 16) return 16;
    return 0;
}

}  // namespace

// (K, MAXD) pairs with K * (MAXD + 2) <= 96 registers of ring state are compiled.
#define ASR_TDT_DISPATCH(LAUNCH, ...)                                            \
    switch (k * 100 + md) {                                                      \
        case 102: return LAUNCH<1, 2>(__VA_ARGS__);                              \
        case 104: return LAUNCH<1, 4>(__VA_ARGS__);                              \
        case 108: return LAUNCH<1, 8>(__VA_ARGS__);                              \
        case 116: return LAUNCH<1, 16>(__VA_ARGS__);                             \
        case 202: return LAUNCH<2, 2>(__VA_ARGS__);                              \
        case 204: return LAUNCH<2, 4>(__VA_ARGS__);                              \
        case 208: return LAUNCH<2, 8>(__VA_ARGS__);                              \
        case 216: return LAUNCH<2, 16>(__VA_ARGS__);                             \
        case 402: return LAUNCH<4, 2>(__VA_ARGS__);                              \
        case 404: return LAUNCH<4, 4>(__VA_ARGS__);                              \
        case 408: return LAUNCH<4, 8>(__VA_ARGS__);                              \
        case 416: return LAUNCH<4, 16>(__VA_ARGS__);                             \
        case 802: return LAUNCH<8, 2>(__VA_ARGS__);                              \
        case 804: return LAUNCH<8, 4>(__VA_ARGS__);                              \
        case 808: return LAUNCH<8, 8>(__VA_ARGS__);                              \
        case 1602: return LAUNCH<16, 2>(__VA_ARGS__);                            \
        case 1604: return LAUNCH<16, 4>(__VA_ARGS__);                            \
        default: return ASR_ERR_UNSUPPORTED;                                     \
    }

int launch_tdt_alpha(const LatticeMeta& m, int B, int U, int max_duration, const int32_t* durations, int n_dur,
                     int has_zero, const float* lpb, const float* lpy, const float* lpd, double* alpha,
                     float* log_prob, float* loss, cudaStream_t st) {
    if (n_dur < 1 || n_dur > kTdtMaxDurClasses) return ASR_ERR_UNSUPPORTED;
    const int k = dp_lanes_k(U), md = tdt_maxd_bucket(max_duration);
    ASR_TDT_DISPATCH(tdt_alpha_launch, m, B, durations, n_dur, has_zero, lpb, lpy, lpd, alpha, log_prob, loss, st)
}

int launch_tdt_beta(const LatticeMeta& m, int B, int U, int max_duration, const int32_t* durations, int n_dur,
                    int has_zero, const float* lpb, const float* lpy, const float* lpd, const double* alpha,
                    const float* grad_loss, float* cb, float* ct, float* gdur, cudaStream_t st) {
    if (n_dur < 1 || n_dur > kTdtMaxDurClasses) return ASR_ERR_UNSUPPORTED;
    const int k = dp_lanes_k(U), md = tdt_maxd_bucket(max_duration);
    ASR_TDT_DISPATCH(tdt_beta_launch, m, B, durations, n_dur, has_zero, lpb, lpy, lpd, alpha, grad_loss, cb, ct,
                     gdur, st)
}

}  // namespace asr
