// TDT lattice recursions on the (T_b + 1)-frame grid: alpha (forward), beta
// (backward) and the edge posteriors with the duration-head logit gradient.
// Reference semantics: tdt.cu:195-428, tests/loss/tdt_reference.py:109-356.
//
// Every TDT edge leaves node (t, u) on anti-diagonal g = t + u and lands on a
// strictly later diagonal: a blank of duration d lands on g + d (d >= 1) and a
// token of duration d lands on g + d + 1 (d >= 0, so the intra-frame d = 0 chain
// is just a distance-1 edge). One CTA sweeps the diagonals of one utterance with
// one thread per label position u, so a diagonal is one parallel step:
//  * forward (pull): alpha(t, u) = log-sum-exp over its <= 2(MAXD+1) incoming
//    edges, whose sources lie on the previous MAXD+1 diagonals;
//  * backward (pull): beta(t, u) likewise over its outgoing edges.
// The recursion variables of the last MAXD+2 diagonals live in a CTA-wide
// shared-memory ring (float64), so a thread reads its neighbour label position
// directly; one __syncthreads separates consecutive diagonals. Each thread
// fetches the weights of its next node (blank / label / duration log-probs) one
// diagonal ahead into a shared-memory ring, by plain loads into registers when
// the duration classes are unique and by cp.async otherwise, so the
// global-memory latency overlaps the current diagonal. The edge posteriors need alpha and
// beta but feed neither recursion: a separate kernel computes them for all
// nodes in parallel once beta is complete.
// Durations are arbitrary (duplicates allowed): for each duration value the
// matching duration classes form a bit mask and their log-probs are log-summed
// (a direct index when the class is unique, the common case, which has its own
// branch-free path). As in the reference, the d = 0 token chain of the
// recursions uses the first zero-duration class only, while posteriors cover
// every class.
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
    bool uniq;  // no two classes share a duration value (the common case)
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
    d.uniq = true;
#pragma unroll
    for (int dv = 0; dv <= MAXD; ++dv) d.uniq = d.uniq && d.single[dv] != -1;
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
struct DpSmem {
    float* wring;
    double* vring;
};

__host__ __device__ inline size_t dp_smem_bytes(int RW, int RV, int W, int NT) {
    return (size_t)RV * NT * sizeof(double) + (size_t)RW * W * NT * sizeof(float);
}

__device__ __forceinline__ DpSmem carve_dp(void* raw, int RV, int NT) {
    DpSmem s;
    s.vring = reinterpret_cast<double*>(raw);
    s.wring = reinterpret_cast<float*>(reinterpret_cast<char*>(raw) + (size_t)RV * NT * sizeof(double));
    return s;
}

// Register copies of node n's weights (blank, label, duration classes: W <= R
// values) and their store into ring slot `slot`: with unique duration classes
// W <= MAXD + 3, and plain loads issued one diagonal ahead cost the step far
// fewer instructions than per-word cp.async copies.
template <int R>
__device__ __forceinline__ void load_node(float (&w)[R], int W, int n, int n_dur, const float* lpb, const float* lpy,
                                          const float* lpd) {
    const float* src = lpd + (int64_t)n * n_dur;
#pragma unroll
    for (int k = 0; k < R; ++k)
        if (k < W) w[k] = k == 0 ? __ldg(lpb + n) : (k == 1 ? __ldg(lpy + n) : __ldg(src + k - 2));
}
template <int R>
__device__ __forceinline__ void store_node(const DpSmem& s, const float (&w)[R], int slot, int W, int NT, int u) {
    float* dst = s.wring + (size_t)slot * W * NT + u;
#pragma unroll
    for (int k = 0; k < R; ++k)
        if (k < W) dst[k * NT] = w[k];
}

// cp.async copies of node (t, u)'s weights into ring slot `slot`.
__device__ __forceinline__ void prefetch_node(const DpSmem& s, int slot, int W, int NT, int u, int n, int n_dur,
                                              const float* lpb, const float* lpy, const float* lpd) {
    float* dst = s.wring + (size_t)slot * W * NT + u;
    cp_async4(dst, lpb + n);
    cp_async4(dst + NT, lpy + n);
    const float* src = lpd + (int64_t)n * n_dur;
    for (int k = 0; k < n_dur; ++k) cp_async4(dst + (2 + k) * NT, src + k);
}

// kGW: the edge weights are read from global memory (L1 / L2) at the source
// nodes instead of from the shared-memory weight ring, so a label position costs
// only its alpha ring in shared memory: the variant for label axes whose ring
// would not fit (U above about 830 with five duration classes).
template <int MAXD, bool kGW>
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
    const DpSmem s = carve_dp(dp_raw, RV, NT);
    const DurTable<MAXD> dt = make_dur_table<MAXD>(durations, n_dur, has_zero);
    const int Tb = m.Tb[b], Ub = m.Ub[b], off = m.off[b], aoff = m.aoff[b];
    const bool lane_in = u < Ub;
    for (int i = u; i < RV * NT; i += NT) s.vring[i] = kNeg;

    const int last = Tb + Ub - 1;
    // Weights one diagonal ahead: registers stored into the ring (unique classes),
    // else cp.async copies. Diagonal 0 is node (0, 0) only.
    float wreg[MAXD + 3];
    bool have = u == 0 && Tb > 0;
    if (!kGW) {
        if (dt.uniq) {
            if (have) load_node(wreg, W, off, n_dur, lpb, lpy, lpd);
        } else {
            if (have) prefetch_node(s, 0, W, NT, 0, off, n_dur, lpb, lpy, lpd);
            cp_async_commit();
        }
    }
    for (int g = 0; g <= last; ++g) {
        const int t1 = g + 1 - u;
        const bool next = g < last && lane_in && t1 >= 0 && t1 < Tb;
        if (kGW) {
        } else if (dt.uniq) {
            if (have) store_node(s, wreg, g % RW, W, NT, u);  // diagonal g, read from g + 1 on
            if (next) load_node(wreg, W, off + t1 * Ub + u, n_dur, lpb, lpy, lpd);
            have = next;
        } else {
            if (next) prefetch_node(s, (g + 1) % RW, W, NT, u, off + t1 * Ub + u, n_dur, lpb, lpy, lpd);
            cp_async_commit();
            cp_async_wait_prev();
        }
        __syncthreads();  // weights of diagonal g and alpha of diagonal g - 1 are visible
        const int t = g - u;
        if (lane_in && t >= 0 && t <= Tb) {
            double a;
            if (t == 0 && u == 0) {
                a = 0.0;
            } else if (dt.uniq) {
                // Unique duration classes: every operand is read from the rings
                // unconditionally (all the slots addressed hold earlier diagonals,
                // see RW / RV) and the invalid terms are dropped by selects, so
                // the node's shared-memory reads overlap instead of each waiting
                // behind its own branch.
                const int ul = u >= 1 ? u - 1 : 0;
                float wsum[2 * (MAXD + 1)];
                double vsrc[2 * (MAXD + 1)];
#pragma unroll
                for (int dv = 0; dv <= MAXD; ++dv) {
                    const int kb = max(dt.single[dv], 0);
                    const int kt = max(dv == 0 ? dt.tok0_k : dt.single[dv], 0);
                    if (kGW) {  // source rows clamped into the utterance; invalid terms are dropped below
                        const int ts = min(max(t - dv, 0), Tb - 1);
                        const int nb = off + ts * Ub + u, nt = off + ts * Ub + ul;
                        wsum[dv] = __ldg(lpb + nb) + __ldg(lpd + (int64_t)nb * n_dur + kb);
                        wsum[MAXD + 1 + dv] = __ldg(lpy + nt) + __ldg(lpd + (int64_t)nt * n_dur + kt);
                    } else {
                        const float* wb = s.wring + (size_t)((g - dv + RW) % RW) * W * NT + u;       // (t - dv, u)
                        const float* wt = s.wring + (size_t)((g - dv - 1 + RW) % RW) * W * NT + ul;  // (t - dv, u - 1)
                        wsum[dv] = wb[0] + wb[(2 + kb) * NT];
                        wsum[MAXD + 1 + dv] = wt[NT] + wt[(2 + kt) * NT];
                    }
                    vsrc[dv] = s.vring[((g - dv + RV) % RV) * NT + u];
                    vsrc[MAXD + 1 + dv] = s.vring[((g - dv - 1 + RV) % RV) * NT + ul];
                }
                double terms[2 * (MAXD + 1)];
#pragma unroll
                for (int dv = 0; dv <= MAXD; ++dv) {
                    const bool src_in = t - dv >= 0 && t - dv < Tb;
                    const int kt = dv == 0 ? dt.tok0_k : dt.single[dv];
                    terms[dv] = (dv >= 1 && dt.single[dv] >= 0 && src_in) ? vsrc[dv] + (double)wsum[dv]
                                                                           : (double)kNeg;
                    terms[MAXD + 1 + dv] = (u >= 1 && kt >= 0 && src_in)
                                               ? vsrc[MAXD + 1 + dv] + (double)wsum[MAXD + 1 + dv]
                                               : (double)kNeg;
                }
                a = lse_d(terms);
            } else {
                double terms[2 * (MAXD + 1)];
#pragma unroll
                for (int i = 0; i < 2 * (MAXD + 1); ++i) terms[i] = kNeg;
                // blank (t - d, u) -> (t, u), d >= 1: source on diagonal g - d
#pragma unroll
                for (int dv = 1; dv <= MAXD; ++dv) {
                    if (dt.mask[dv] && t - dv >= 0 && t - dv < Tb) {
                        float e;
                        if (kGW) {
                            const int n = off + (t - dv) * Ub + u;
                            e = __ldg(lpb + n) + dur_weight(lpd + (int64_t)n * n_dur, 1, dt.mask[dv], dt.single[dv]);
                        } else {
                            const float* w = s.wring + (size_t)((g - dv) % RW) * W * NT + u;
                            e = w[0] + dur_weight(w + 2 * NT, NT, dt.mask[dv], dt.single[dv]);
                        }
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
                            float e;
                            if (kGW) {
                                const int n = off + (t - dv) * Ub + (u - 1);
                                e = __ldg(lpy + n) + dur_weight(lpd + (int64_t)n * n_dur, 1, mk, sk);
                            } else {
                                const float* w = s.wring + (size_t)((g - dv - 1) % RW) * W * NT + (u - 1);
                                e = w[NT] + dur_weight(w + 2 * NT, NT, mk, sk);
                            }
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

// beta(t, u) for t <= T_b (same layout as alpha). Only the recursion runs here,
// one diagonal per step; the edge posteriors, which do not feed the recursion,
// are computed afterwards for all nodes at once by tdt_posterior_kernel, so the
// serial diagonal chain carries the log-sum-exp alone.
template <int MAXD>
__global__ void tdt_beta_kernel(LatticeMeta m, int n_threads, const int32_t* __restrict__ durations, int n_dur,
                                int has_zero, const float* __restrict__ lpb, const float* __restrict__ lpy,
                                const float* __restrict__ lpd, double* __restrict__ beta) {
    constexpr int RW = 2;         // weights of diagonals g and g - 1 (each thread reads only its own column)
    constexpr int RV = MAXD + 2;  // beta of diagonals g .. g + MAXD + 1
    extern __shared__ __align__(16) unsigned char dp_raw[];
    const int NT = n_threads, W = 2 + n_dur;
    const int u = threadIdx.x;
    const int b = blockIdx.x;
    const DpSmem s = carve_dp(dp_raw, RV, NT);
    const DurTable<MAXD> dt = make_dur_table<MAXD>(durations, n_dur, has_zero);
    const int Tb = m.Tb[b], Ub = m.Ub[b], off = m.off[b], aoff = m.aoff[b];
    const bool lane_in = u < Ub;
    for (int i = u; i < RV * NT; i += NT) s.vring[i] = kNeg;

    const int first = Tb + Ub - 1;
    // The node's own weights one diagonal ahead: registers stored into the ring
    // (unique classes), else cp.async copies.
    auto node_in = [&](int g) {
        const int t = g - u;
        return g >= 0 && lane_in && t >= 0 && t < Tb;
    };
    float wreg[MAXD + 3];
    bool have = node_in(first);
    if (dt.uniq) {
        if (have) load_node(wreg, W, off + (first - u) * Ub + u, n_dur, lpb, lpy, lpd);
    } else {
        if (have) prefetch_node(s, first & 1, W, NT, u, off + (first - u) * Ub + u, n_dur, lpb, lpy, lpd);
        cp_async_commit();
    }
    for (int g = first; g >= 0; --g) {
        const bool next = node_in(g - 1);
        if (dt.uniq) {
            if (have) store_node(s, wreg, g & 1, W, NT, u);
            if (next) load_node(wreg, W, off + (g - 1 - u) * Ub + u, n_dur, lpb, lpy, lpd);
            have = next;
        } else {
            if (next) prefetch_node(s, (g - 1) & 1, W, NT, u, off + (g - 1 - u) * Ub + u, n_dur, lpb, lpy, lpd);
            cp_async_commit();
            cp_async_wait_prev();
        }
        __syncthreads();  // weights of diagonal g and beta of diagonal g + 1 are visible
        const int t = g - u;
        double be = kNeg;
        if (lane_in && t >= 0 && t <= Tb) {
            if (t == Tb) {
                be = (u == Ub - 1) ? 0.0 : (double)kNeg;  // terminal seed (tdt.cu:331,351)
            } else {
                const float* w = s.wring + (size_t)(g & 1) * W * NT + u;
                const float lb = w[0], ly = w[NT];
                const bool can_tok = u < Ub - 1;
                double terms[2 * (MAXD + 1)];
                if (dt.uniq) {
                    // Unique duration classes: every operand is read unconditionally
                    // and invalid terms are selected away, so the reads overlap.
                    const int ur = u + 1 < NT ? u + 1 : u;
                    float ldv[MAXD + 1];
                    double bown[MAXD + 1], bnext[MAXD + 1];
#pragma unroll
                    for (int dv = 0; dv <= MAXD; ++dv) {
                        ldv[dv] = w[(2 + max(dt.single[dv], 0)) * NT];
                        bown[dv] = s.vring[((g + dv) % RV) * NT + u];
                        bnext[dv] = s.vring[((g + dv + 1) % RV) * NT + ur];
                    }
                    const float ld0 = w[(2 + max(dt.tok0_k, 0)) * NT];  // the d = 0 token chain's class
#pragma unroll
                    for (int dv = 0; dv <= MAXD; ++dv) {
                        const bool dst_in = t + dv <= Tb;
                        const int kt = dv == 0 ? dt.tok0_k : dt.single[dv];
                        terms[dv] = (dv >= 1 && dt.single[dv] >= 0 && dst_in) ? bown[dv] + (double)(lb + ldv[dv])
                                                                               : (double)kNeg;
                        terms[MAXD + 1 + dv] = (can_tok && kt >= 0 && dst_in)
                                                   ? bnext[dv] + (double)(ly + (dv == 0 ? ld0 : ldv[dv]))
                                                   : (double)kNeg;
                    }
                } else {
                    const float* ld = w + 2 * NT;
#pragma unroll
                    for (int i = 0; i < 2 * (MAXD + 1); ++i) terms[i] = kNeg;
#pragma unroll
                    for (int dv = 1; dv <= MAXD; ++dv)
                        if (dt.mask[dv] && t + dv <= Tb)
                            terms[dv] = s.vring[((g + dv) % RV) * NT + u] +
                                        (double)(lb + dur_weight(ld, NT, dt.mask[dv], dt.single[dv]));
                    if (can_tok) {
#pragma unroll
                        for (int dv = 0; dv <= MAXD; ++dv) {
                            const uint32_t mk = dv == 0 ? dt.tok0 : dt.mask[dv];
                            const int sk = dv == 0 ? dt.tok0_k : dt.single[dv];
                            if (mk && t + dv <= Tb)
                                terms[MAXD + 1 + dv] = s.vring[((g + dv + 1) % RV) * NT + u + 1] +
                                                       (double)(ly + dur_weight(ld, NT, mk, sk));
                        }
                    }
                }
                be = lse_d(terms);
            }
            beta[aoff + t * Ub + u] = be;
        }
        s.vring[(g % RV) * NT + u] = be;
    }
}

// Edge posteriors of every node (t < T_b, u < U_b) from alpha and beta, one
// thread per node (grid-stride): cb = gl * blank posterior, ct = gl * token
// posterior (both summed over durations) and gdur[k] = d loss / d duration-logit k
// (tdt.cu:400-426 + 475-500). Posteriors cover every duration class, including
// zero-duration classes other than the one the d = 0 token chain uses.
template <int MAXD>
__global__ void __launch_bounds__(256) tdt_posterior_kernel(
    LatticeMeta m, int B, const int32_t* __restrict__ durations, int n_dur, int has_zero,
    const float* __restrict__ lpb, const float* __restrict__ lpy, const float* __restrict__ lpd,
    const double* __restrict__ alpha, const double* __restrict__ beta, const float* __restrict__ grad_loss,
    float* __restrict__ cb, float* __restrict__ ct, float* __restrict__ gdur) {
    const DurTable<MAXD> dt = make_dur_table<MAXD>(durations, n_dur, has_zero);
    const int N = total_nodes(m, B);
    for (int n = blockIdx.x * blockDim.x + threadIdx.x; n < N; n += gridDim.x * blockDim.x) {
        const NodeCoord c = node_coord(m, B, n);
        const int Tb = __ldg(m.Tb + c.b), Ub = c.Ub, t = c.t, u = c.u;
        const int aoff = __ldg(m.aoff + c.b);
        const double logZ = alpha[aoff + Tb * Ub + Ub - 1];  // exact-landing terminal, float64
        const float gl = __ldg(grad_loss + c.b);
        const double a = alpha[aoff + t * Ub + u];
        const float lb = __ldg(lpb + n), ly = __ldg(lpy + n);
        const float* ld = lpd + (int64_t)n * n_dur;
        const bool can_tok = u < Ub - 1;
        const double* bo = beta + aoff + u;  // beta(t', u) = bo[t' * Ub]
        double bown[MAXD + 1], bnext[MAXD + 1];
#pragma unroll
        for (int dv = 0; dv <= MAXD; ++dv) {
            const bool in = t + dv <= Tb;
            bown[dv] = in ? bo[(t + dv) * Ub] : (double)kNeg;
            bnext[dv] = (in && can_tok) ? bo[(t + dv) * Ub + 1] : (double)kNeg;
        }
        const double ab = a + (double)lb - logZ, at = a + (double)ly - logZ;
        float bp = 0.f, tp = 0.f;
        float* gd = gdur + (int64_t)n * n_dur;
        if (dt.uniq) {
            float gk[MAXD + 1], ldv[MAXD + 1];
            float gsum = 0.f;
#pragma unroll
            for (int dv = 0; dv <= MAXD; ++dv) {
                ldv[dv] = dt.single[dv] >= 0 ? __ldg(ld + dt.single[dv]) : 0.f;
                const bool on = dt.single[dv] >= 0 && t + dv <= Tb;
                const float gbk = (on && dv >= 1) ? __expf((float)(ab + bown[dv]) + ldv[dv]) : 0.f;
                const float gtk = (on && can_tok) ? __expf((float)(at + bnext[dv]) + ldv[dv]) : 0.f;
                bp += gbk;
                tp += gtk;
                gk[dv] = -(gbk + gtk);
                gsum += gk[dv];
            }
#pragma unroll
            for (int dv = 0; dv <= MAXD; ++dv)
                if (dt.single[dv] >= 0) gd[dt.single[dv]] = gl * (gk[dv] - __expf(ldv[dv]) * gsum);
        } else {
            float gi[kTdtMaxDurClasses];
            for (int k = 0; k < n_dur; ++k) gi[k] = 0.f;
#pragma unroll
            for (int dv = 0; dv <= MAXD; ++dv) {
                if (t + dv > Tb) continue;
                uint32_t mk = dt.mask[dv];
                const float base_b = (dv >= 1) ? (float)(ab + bown[dv]) : -INFINITY;
                const float base_t = can_tok ? (float)(at + bnext[dv]) : -INFINITY;
                while (mk) {
                    const int k = __ffs(mk) - 1;
                    mk &= mk - 1;
                    const float x = __ldg(ld + k);
                    const float gbk = (dv >= 1) ? __expf(base_b + x) : 0.f;
                    const float gtk = can_tok ? __expf(base_t + x) : 0.f;
                    bp += gbk;
                    tp += gtk;
                    gi[k] = -(gbk + gtk);
                }
            }
            float gsum = 0.f;
            for (int k = 0; k < n_dur; ++k) gsum += gi[k];
            for (int k = 0; k < n_dur; ++k) gd[k] = gl * (gi[k] - __expf(__ldg(ld + k)) * gsum);
        }
        cb[n] = gl * bp;
        ct[n] = gl * tp;
    }
}

// One CTA of NT threads per utterance must fit the SM's register file; wider
// duration rings (MAXD 8, 16) use more registers per thread and so cap the label
// axis lower than 1024 (a clean ASR_ERR_UNSUPPORTED instead of a failed launch).
template <typename Kern>
bool fits_registers(Kern k, int NT) {
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, k) != cudaSuccess) return false;
    const int regs = (fa.numRegs + 7) / 8 * 8;  // per-thread allocation granularity
    return NT <= fa.maxThreadsPerBlock && (int64_t)regs * NT <= 65536;
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
    const size_t smem = dp_smem_bytes(MAXD + 4, MAXD + 2, 2 + nd, NT);
    KernelTimer kt("tdt_alpha", st);
    if (smem <= 227 * 1024) {  // weights in the shared-memory ring
        if (!fits_registers(tdt_alpha_kernel<MAXD, false>, NT) || set_smem(tdt_alpha_kernel<MAXD, false>, smem))
            return ASR_ERR_UNSUPPORTED;
        tdt_alpha_kernel<MAXD, false><<<B, NT, smem, st>>>(m, NT, dur, nd, hz, lpb, lpy, lpd, alpha, lp, loss);
    } else {  // long label axis: weights read at the source nodes, alpha ring only
        const size_t smem_g = dp_smem_bytes(0, MAXD + 2, 2 + nd, NT);
        if (!fits_registers(tdt_alpha_kernel<MAXD, true>, NT) || set_smem(tdt_alpha_kernel<MAXD, true>, smem_g))
            return ASR_ERR_UNSUPPORTED;
        tdt_alpha_kernel<MAXD, true><<<B, NT, smem_g, st>>>(m, NT, dur, nd, hz, lpb, lpy, lpd, alpha, lp, loss);
    }
    ASR_LAUNCH_CHECK();
    return ASR_OK;
}

template <int MAXD>
int tdt_beta_launch(const LatticeMeta& m, int B, int U, const int32_t* dur, int nd, int hz, const float* lpb,
                    const float* lpy, const float* lpd, const double* alpha, const float* gl, float* cb, float* ct,
                    float* gdur, double* beta, cudaStream_t st) {
    const int NT = dp_threads(U);
    const size_t smem = dp_smem_bytes(2, MAXD + 2, 2 + nd, NT);
    if (!fits_registers(tdt_beta_kernel<MAXD>, NT) || set_smem(tdt_beta_kernel<MAXD>, smem))
        return ASR_ERR_UNSUPPORTED;
    {
        KernelTimer kt("tdt_beta", st);
        tdt_beta_kernel<MAXD><<<B, NT, smem, st>>>(m, NT, dur, nd, hz, lpb, lpy, lpd, beta);
        ASR_LAUNCH_CHECK();
    }
    KernelTimer kt("tdt_posteriors", st);
    tdt_posterior_kernel<MAXD><<<sm_count() * 8, 256, 0, st>>>(m, B, dur, nd, hz, lpb, lpy, lpd, alpha, beta, gl, cb,
                                                               ct, gdur);
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
                    const float* grad_loss, float* cb, float* ct, float* gdur, double* beta, cudaStream_t st) {
    if (n_dur < 1 || n_dur > kTdtMaxDurClasses || U > 1024) return ASR_ERR_UNSUPPORTED;
    const int md = tdt_maxd_bucket(max_duration);
    ASR_TDT_DISPATCH(tdt_beta_launch, m, B, U, durations, n_dur, has_zero, lpb, lpy, lpd, alpha, grad_loss, cb, ct,
                     gdur, beta, st)
}

}  // namespace asr
