// TDT lattice recursions on the (T_b + 1)-frame grid: alpha (forward) and beta
// fused with the edge posteriors and the duration-head logit gradient
// (backward). Reference semantics: tdt.cu:195-428, tests/loss/tdt_reference.py:109-356.
//
// Every TDT edge leaves node (t, u) on anti-diagonal g = t + u and lands on a
// strictly later diagonal: a blank of duration d lands on g + d (d >= 1) and a
// token of duration d lands on g + d + 1 (d >= 0, so the intra-frame d = 0 chain
// is just a distance-1 edge). One CTA sweeps the diagonals of one utterance with
// one thread per label position u, so a diagonal is one parallel step:
//  * forward (pull): alpha(t, u) = log-sum-exp over its <= 2(MAXD+1) incoming
//    edges, whose sources lie on the previous MAXD+1 diagonals;
//  * backward (pull): beta(t, u) likewise over its outgoing edges, and the same
//    terms give every edge posterior of (t, u) in place.
// The recursion variables of the last MAXD+2 diagonals live in a CTA-wide
// shared-memory ring (float64), so a thread reads its neighbour label position
// directly; one __syncthreads separates consecutive diagonals. Each thread
// copies the weights of its next node (blank / label / duration log-probs, and
// alpha in the backward) into a shared-memory ring with cp.async one diagonal
// ahead, so the global-memory latency overlaps the current diagonal.
// Durations are arbitrary (duplicates allowed): for each duration value the
// matching duration classes form a bit mask and their log-probs are log-summed
// (a direct index when the class is unique, the common case). As in the
// reference, the d = 0 token chain of the recursions uses the first zero-duration
// class only, while posteriors cover every class.
#include <algorithm>

#include "dp.cuh"

namespace asr {
namespace {

// Duration classes per duration value dv: a bit mask and, when exactly one class
// has that value, its index (-1 otherwise; -2 when none).
template <int MAXD>
struct DurTable {
    uint32_t mask[MAXD + 1];
    int single[MAXD + 1];
    uint32_t tok0;  // class used by the d = 0 token chain (first zero duration)
    int tok0_k;
};

template <int MAXD>
__device__ __forceinline__ DurTable<MAXD> make_dur_table(const int32_t* __restrict__ durations, int n_dur,
                                                         int has_zero) {
    DurTable<MAXD> d;
#pragma unroll
    for (int dv = 0; dv <= MAXD; ++dv) d.mask[dv] = 0u;
    int zk = -1;
    for (int k = 0; k < n_dur; ++k) {
        const int dk = durations[k];
#pragma unroll
        for (int dv = 0; dv <= MAXD; ++dv)
            if (dk == dv) d.mask[dv] |= 1u << k;
        if (dk == 0 && zk < 0) zk = k;
    }
#pragma unroll
    for (int dv = 0; dv <= MAXD; ++dv)
        d.single[dv] = d.mask[dv] == 0u ? -2 : (__popc(d.mask[dv]) == 1 ? __ffs(d.mask[dv]) - 1 : -1);
    d.tok0 = (has_zero && zk >= 0) ? (1u << zk) : 0u;
    d.tok0_k = (has_zero && zk >= 0) ? zk : -2;
    return d;
}

// Log-sum of the duration log-probs of the classes in `mask` (ld[k * stride]).
__device__ __forceinline__ float dur_weight(const float* ld, int stride, uint32_t mask, int single) {
    if (single >= 0) return ld[single * stride];
    float w = kNeg;
    bool first = true;
    while (mask) {
        const int k = __ffs(mask) - 1;
        mask &= mask - 1;
        const float x = ld[k * stride];
        w = first ? x : lae(w, x);
        first = false;
    }
    return w;
}

// Shared memory of one CTA (NT = blockDim.x threads, one per label position):
//   wring[RW][W][NT]  node weights: [0] blank, [1] label, [2 + k] duration k
//   vring[RV][NT]     recursion variable (alpha or beta) of recent diagonals, float64
//   aslot[2][NT]      alpha of the node being processed (backward only), float64
//   gi[n_dur][NT]     per-class duration-log-prob gradient (backward only)
struct DpSmem {
    float* wring;
    double* vring;
    double* aslot;
    float* gi;
};

__host__ __device__ inline size_t dp_smem_bytes(int RW, int RV, int W, int NT, int n_dur, bool bwd) {
    size_t b = (size_t)RV * NT * sizeof(double) + (size_t)RW * W * NT * sizeof(float);
    if (bwd) b += 2 * (size_t)NT * sizeof(double) + (size_t)n_dur * NT * sizeof(float);
    return b;
}

__device__ __forceinline__ DpSmem carve_dp(void* raw, int RW, int RV, int W, int NT, int n_dur, bool bwd) {
    DpSmem s;
    char* p = reinterpret_cast<char*>(raw);
    s.vring = reinterpret_cast<double*>(p);
    p += (size_t)RV * NT * sizeof(double);
    s.aslot = bwd ? reinterpret_cast<double*>(p) : nullptr;
    if (bwd) p += 2 * (size_t)NT * sizeof(double);
    s.wring = reinterpret_cast<float*>(p);
    p += (size_t)RW * W * NT * sizeof(float);
    s.gi = bwd ? reinterpret_cast<float*>(p) : nullptr;
    return s;
}

// cp.async copies of node (t, u)'s weights into ring slot `slot` (and its alpha).
__device__ __forceinline__ void prefetch_node(const DpSmem& s, int slot, int W, int NT, int u, int n, int n_dur,
                                              const float* lpb, const float* lpy, const float* lpd,
                                              const double* alpha_src, int aslot) {
    float* dst = s.wring + (size_t)slot * W * NT + u;
    cp_async4(dst, lpb + n);
    cp_async4(dst + NT, lpy + n);
    const float* src = lpd + (int64_t)n * n_dur;
    for (int k = 0; k < n_dur; ++k) cp_async4(dst + (2 + k) * NT, src + k);
    if (alpha_src) cp_async8(s.aslot + aslot * NT + u, alpha_src);
}

template <int MAXD>
__global__ void tdt_alpha_kernel(LatticeMeta m, int n_threads, const int32_t* __restrict__ durations, int n_dur,
                                 int has_zero, const float* __restrict__ lpb, const float* __restrict__ lpy,
                                 const float* __restrict__ lpd, double* __restrict__ alpha,
                                 float* __restrict__ log_prob, float* __restrict__ loss) {
    // Weights of diagonals g - MAXD - 2 .. g + 1. Token edges read the left
    // neighbour's column; the extra slot keeps the next prefetch (issued before
    // the diagonal barrier) away from the oldest slot a slower thread may still
    // read in the previous iteration.
    constexpr int RW = MAXD + 4;
    constexpr int RV = MAXD + 2;  // alpha of diagonals g - MAXD - 1 .. g
    extern __shared__ __align__(16) unsigned char dp_raw[];
    const int NT = n_threads, W = 2 + n_dur;
    const int u = threadIdx.x;
    const int b = blockIdx.x;
    const DpSmem s = carve_dp(dp_raw, RW, RV, W, NT, n_dur, false);
    const DurTable<MAXD> dt = make_dur_table<MAXD>(durations, n_dur, has_zero);
    const int Tb = m.Tb[b], Ub = m.Ub[b], off = m.off[b], aoff = m.aoff[b];
    const bool lane_in = u < Ub;
    for (int i = u; i < RV * NT; i += NT) s.vring[i] = kNeg;

    const int last = Tb + Ub - 1;
    // prefetch diagonal 0: node (0, 0) only
    if (u == 0 && Tb > 0) prefetch_node(s, 0, W, NT, 0, off, n_dur, lpb, lpy, lpd, nullptr, 0);
    cp_async_commit();
    for (int g = 0; g <= last; ++g) {
        {
            const int t1 = g + 1 - u;
            if (g < last && lane_in && t1 >= 0 && t1 < Tb)
                prefetch_node(s, (g + 1) % RW, W, NT, u, off + t1 * Ub + u, n_dur, lpb, lpy, lpd, nullptr, 0);
            cp_async_commit();
        }
        cp_async_wait_prev();
        __syncthreads();  // weights of diagonal g and alpha of diagonal g - 1 are visible
        const int t = g - u;
        if (lane_in && t >= 0 && t <= Tb) {
            double a;
            if (t == 0 && u == 0) {
                a = 0.0;
            } else {
                double terms[2 * (MAXD + 1)];
#pragma unroll
                for (int i = 0; i < 2 * (MAXD + 1); ++i) terms[i] = kNeg;
                // blank (t - d, u) -> (t, u), d >= 1: source on diagonal g - d
#pragma unroll
                for (int dv = 1; dv <= MAXD; ++dv) {
                    if (dt.mask[dv] && t - dv >= 0 && t - dv < Tb) {
                        const float* w = s.wring + (size_t)((g - dv) % RW) * W * NT + u;
                        const float e = w[0] + dur_weight(w + 2 * NT, NT, dt.mask[dv], dt.single[dv]);
                        terms[dv] = s.vring[((g - dv) % RV) * NT + u] + (double)e;
                    }
                }
                // token (t - d, u - 1) -> (t, u), d >= 0: source on diagonal g - d - 1
                if (u >= 1) {
#pragma unroll
                    for (int dv = 0; dv <= MAXD; ++dv) {
                        const uint32_t mk = dv == 0 ? dt.tok0 : dt.mask[dv];
                        const int sk = dv == 0 ? dt.tok0_k : dt.single[dv];
                        if (mk && t - dv >= 0 && t - dv < Tb) {
                            const float* w = s.wring + (size_t)((g - dv - 1) % RW) * W * NT + (u - 1);
                            const float e = w[NT] + dur_weight(w + 2 * NT, NT, mk, sk);
                            terms[MAXD + 1 + dv] = s.vring[((g - dv - 1) % RV) * NT + u - 1] + (double)e;
                        }
                    }
                }
                a = lse_d(terms);
            }
            s.vring[(g % RV) * NT + u] = a;
            alpha[aoff + t * Ub + u] = a;
            if (t == Tb && u == Ub - 1) {  // exact-landing terminal (tdt.cu:291-295)
                log_prob[b] = (float)a;
                loss[b] = (float)(-a);
            }
        } else {
            s.vring[(g % RV) * NT + u] = kNeg;
        }
    }
}

// Writes per node: cb = gl * blank posterior, ct = gl * token posterior (both summed
// over durations) and gdur[k] = d loss / d duration-logit k (tdt.cu:400-426 + 475-500).
template <int MAXD>
__global__ void tdt_beta_kernel(LatticeMeta m, int n_threads, const int32_t* __restrict__ durations, int n_dur,
                                int has_zero, const float* __restrict__ lpb, const float* __restrict__ lpy,
                                const float* __restrict__ lpd, const double* __restrict__ alpha,
                                const float* __restrict__ grad_loss, float* __restrict__ cb, float* __restrict__ ct,
                                float* __restrict__ gdur) {
    constexpr int RW = 2;         // weights of diagonals g and g - 1 (each thread reads only its own column)
    constexpr int RV = MAXD + 2;  // beta of diagonals g .. g + MAXD + 1
    extern __shared__ __align__(16) unsigned char dp_raw[];
    const int NT = n_threads, W = 2 + n_dur;
    const int u = threadIdx.x;
    const int b = blockIdx.x;
    const DpSmem s = carve_dp(dp_raw, RW, RV, W, NT, n_dur, true);
    const DurTable<MAXD> dt = make_dur_table<MAXD>(durations, n_dur, has_zero);
    const int Tb = m.Tb[b], Ub = m.Ub[b], off = m.off[b], aoff = m.aoff[b];
    const double logZ = alpha[aoff + Tb * Ub + Ub - 1];  // exact-landing terminal, float64
    const float gl = grad_loss[b];
    const bool lane_in = u < Ub;
    for (int i = u; i < RV * NT; i += NT) s.vring[i] = kNeg;
    float* gi = s.gi + u;  // stride NT

    const int first = Tb + Ub - 1;
    auto prefetch = [&](int g) {
        const int t = g - u;
        if (g >= 0 && lane_in && t >= 0 && t < Tb)
            prefetch_node(s, g & 1, W, NT, u, off + t * Ub + u, n_dur, lpb, lpy, lpd, alpha + aoff + t * Ub + u,
                          g & 1);
        cp_async_commit();
    };
    prefetch(first);
    for (int g = first; g >= 0; --g) {
        prefetch(g - 1);
        cp_async_wait_prev();
        __syncthreads();  // weights of diagonal g and beta of diagonal g + 1 are visible
        const int t = g - u;
        double be = kNeg;
        if (lane_in && t >= 0 && t <= Tb) {
            if (t == Tb) {
                be = (u == Ub - 1) ? 0.0 : (double)kNeg;  // terminal seed (tdt.cu:331,351)
            } else {
                const int n = off + t * Ub + u;
                const float* w = s.wring + (size_t)(g & 1) * W * NT + u;
                const float lb = w[0], ly = w[NT];
                const float* ld = w + 2 * NT;
                const double a = s.aslot[(g & 1) * NT + u];
                const bool can_tok = u < Ub - 1;
                // successor beta values: own position on diagonal g + d, next position on g + d + 1
                double bown[MAXD + 1], bnext[MAXD + 1];
#pragma unroll
                for (int dv = 0; dv <= MAXD; ++dv) {
                    bown[dv] = s.vring[((g + dv) % RV) * NT + u];
                    bnext[dv] = can_tok ? s.vring[((g + dv + 1) % RV) * NT + u + 1] : (double)kNeg;
                }
                double terms[2 * (MAXD + 1)];
#pragma unroll
                for (int i = 0; i < 2 * (MAXD + 1); ++i) terms[i] = kNeg;
#pragma unroll
                for (int dv = 1; dv <= MAXD; ++dv)
                    if (dt.mask[dv] && t + dv <= Tb)
                        terms[dv] = bown[dv] + (double)(lb + dur_weight(ld, NT, dt.mask[dv], dt.single[dv]));
                if (can_tok) {
#pragma unroll
                    for (int dv = 0; dv <= MAXD; ++dv) {
                        const uint32_t mk = dv == 0 ? dt.tok0 : dt.mask[dv];
                        const int sk = dv == 0 ? dt.tok0_k : dt.single[dv];
                        if (mk && t + dv <= Tb)
                            terms[MAXD + 1 + dv] = bnext[dv] + (double)(ly + dur_weight(ld, NT, mk, sk));
                    }
                }
                be = lse_d(terms);
                // edge posteriors of (t, u), every duration class
                for (int k = 0; k < n_dur; ++k) gi[k * NT] = 0.f;
                float bp = 0.f, tp = 0.f;
                const double ab = a + (double)lb - logZ, at = a + (double)ly - logZ;
#pragma unroll
                for (int dv = 0; dv <= MAXD; ++dv) {
                    if (t + dv > Tb) continue;
                    uint32_t mk = dt.mask[dv];
                    const float base_b = (dv >= 1) ? (float)(ab + bown[dv]) : -INFINITY;
                    const float base_t = can_tok ? (float)(at + bnext[dv]) : -INFINITY;
                    while (mk) {
                        const int k = __ffs(mk) - 1;
                        mk &= mk - 1;
                        const float x = ld[k * NT];
                        const float gbk = (dv >= 1) ? __expf(base_b + x) : 0.f;
                        const float gtk = can_tok ? __expf(base_t + x) : 0.f;
                        bp += gbk;
                        tp += gtk;
                        gi[k * NT] = -(gbk + gtk);
                    }
                }
                float gsum = 0.f;
                for (int k = 0; k < n_dur; ++k) gsum += gi[k * NT];
                float* gd = gdur + (int64_t)n * n_dur;
                for (int k = 0; k < n_dur; ++k) gd[k] = gl * (gi[k * NT] - __expf(ld[k * NT]) * gsum);
                cb[n] = gl * bp;
                ct[n] = gl * tp;
            }
        }
        s.vring[(g % RV) * NT + u] = be;
    }
}

template <typename Kern>
int set_smem(Kern k, size_t bytes) {
    if (bytes > 227 * 1024) return ASR_ERR_UNSUPPORTED;
    if (bytes > 48 * 1024 &&
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) != cudaSuccess)
        return ASR_ERR_UNSUPPORTED;
    return ASR_OK;
}

int dp_threads(int U) { return (U + 31) / 32 * 32; }

template <int MAXD>
int tdt_alpha_launch(const LatticeMeta& m, int B, int U, const int32_t* dur, int nd, int hz, const float* lpb,
                     const float* lpy, const float* lpd, double* alpha, float* lp, float* loss, cudaStream_t st) {
    const int NT = dp_threads(U);
    const size_t smem = dp_smem_bytes(MAXD + 4, MAXD + 2, 2 + nd, NT, nd, false);
    if (set_smem(tdt_alpha_kernel<MAXD>, smem)) return ASR_ERR_UNSUPPORTED;
    KernelTimer kt("tdt_alpha", st);
    tdt_alpha_kernel<MAXD><<<B, NT, smem, st>>>(m, NT, dur, nd, hz, lpb, lpy, lpd, alpha, lp, loss);
    ASR_LAUNCH_CHECK();
    return ASR_OK;
}

template <int MAXD>
int tdt_beta_launch(const LatticeMeta& m, int B, int U, const int32_t* dur, int nd, int hz, const float* lpb,
                    const float* lpy, const float* lpd, const double* alpha, const float* gl, float* cb, float* ct,
                    float* gdur, cudaStream_t st) {
    const int NT = dp_threads(U);
    const size_t smem = dp_smem_bytes(2, MAXD + 2, 2 + nd, NT, nd, true);
    if (set_smem(tdt_beta_kernel<MAXD>, smem)) return ASR_ERR_UNSUPPORTED;
    KernelTimer kt("tdt_beta_posteriors", st);
    tdt_beta_kernel<MAXD><<<B, NT, smem, st>>>(m, NT, dur, nd, hz, lpb, lpy, lpd, alpha, gl, cb, ct, gdur);
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

#define ASR_TDT_DISPATCH(LAUNCH, ...)                \
    switch (md) {                                    \
        case 2: return LAUNCH<2>(__VA_ARGS__);       \
        case 4: return LAUNCH<4>(__VA_ARGS__);       \
        case 8: return LAUNCH<8>(__VA_ARGS__);       \
        case 16: return LAUNCH<16>(__VA_ARGS__);     \
        default: return ASR_ERR_UNSUPPORTED;         \
    }

int launch_tdt_alpha(const LatticeMeta& m, int B, int U, int max_duration, const int32_t* durations, int n_dur,
                     int has_zero, const float* lpb, const float* lpy, const float* lpd, double* alpha,
                     float* log_prob, float* loss, cudaStream_t st) {
    if (n_dur < 1 || n_dur > kTdtMaxDurClasses || U > 1024) return ASR_ERR_UNSUPPORTED;
    const int md = tdt_maxd_bucket(max_duration);
    ASR_TDT_DISPATCH(tdt_alpha_launch, m, B, U, durations, n_dur, has_zero, lpb, lpy, lpd, alpha, log_prob, loss, st)
}

int launch_tdt_beta(const LatticeMeta& m, int B, int U, int max_duration, const int32_t* durations, int n_dur,
                    int has_zero, const float* lpb, const float* lpy, const float* lpd, const double* alpha,
                    const float* grad_loss, float* cb, float* ct, float* gdur, cudaStream_t st) {
    if (n_dur < 1 || n_dur > kTdtMaxDurClasses || U > 1024) return ASR_ERR_UNSUPPORTED;
    const int md = tdt_maxd_bucket(max_duration);
    ASR_TDT_DISPATCH(tdt_beta_launch, m, B, U, durations, n_dur, has_zero, lpb, lpy, lpd, alpha, grad_loss, cb, ct,
                     gdur, st)
}

}  // namespace asr
