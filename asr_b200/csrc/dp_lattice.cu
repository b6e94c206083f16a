// Lattice recursions of the RNN-T and TDT losses: alpha (forward), and beta
// with the edge posteriors and the duration-head gradient (backward).
// Reference semantics: rnnt.cu:218-317, tdt.cu:195-500 and the float64 oracles
// tests/loss/rnnt_reference.py:44-259, tests/loss/tdt_reference.py:109-356.
//
// Both recursions run on a grid of T_b + 1 frames and U_b label positions. Every
// edge leaves node (t, u) on anti-diagonal g = t + u for a strictly later one: a
// blank of duration d >= 1 lands on g + d, a token of duration d >= 0 on g + d + 1
// (RNN-T: the blank, d = 1, and the label edge, d = 0). So one CTA per utterance
// sweeps the anti-diagonals, one thread per label position (more positions per
// thread past 512), and a diagonal is one parallel step behind one barrier:
//   forward:  alpha(t, u) = log-sum-exp over its incoming edges (sources on the
//             previous MAXD + 1 diagonals);
//   backward: beta(t, u) likewise over its outgoing edges, then the node's edge
//             posteriors, whose beta values are all on the MAXD + 1 later
//             diagonals already done.
// RNN-T is the TDT recursion with a blank of duration 1 and a label edge of
// duration 0, without a duration head; its terminal x(T_b, U_b - 1) is the final
// blank out of (T_b - 1, U_b - 1).
//
// Layout: the forward joint stores the lattice weights diagonal-major
// (diag_index), and alpha / beta are stored the same way, so each diagonal of
// weights is one contiguous block: it is staged into a shared-memory ring with
// cp.async a few diagonals ahead of its use, every copy coalesced. The
// recursion variables of the last MAXD + 2 diagonals sit in a second ring.
// Label axes too long for those rings (global-memory mode) read the weights
// from global memory and the sources back from the alpha / beta arrays this CTA
// writes.
//
// Arithmetic: the recursion variables reach |x| ~ 10^3, where one fp32 ulp is
// ~1e-4, so they are kept as float pairs hi + lo (about 2^-48 relative). A
// node's log-sum-exp takes the max m of the terms' leading parts, evaluates
// each term's offset ((hi - m) + w) + lo in fp32 (the subtraction is exact
// for the terms that matter), one ex2 per term and one lg2, and stores m + L
// as an exact two-sum. Only fp32 adds and max sit on the dependent chain:
// float64 max and the float64 <-> fp32 conversions each cost ~25 cycles of
// latency here. Edge posteriors subtract log Z the same way.
#include <algorithm>

#include "dp.cuh"

namespace asr {
namespace {

constexpr int kAhead = 2;        // diagonals of weights in flight ahead of their first use (P)
constexpr int kMaxThreads = 512;  // threads per CTA; longer label axes take several positions per thread
constexpr float kLog2e_f = 1.4426950408889634f;
constexpr float kLn2_f = 0.6931471805599453f;

struct Pair {
    float hi, lo;
};

__device__ __forceinline__ Pair two_sum(float a, float b) {
    const float s = a + b;
    const float bb = s - a;
    return {s, (a - (s - bb)) + (b - bb)};
}

__device__ __forceinline__ Pair to_pair(double x) {
    const float hi = (float)x;
    return {hi, (float)(x - (double)hi)};
}

__device__ __forceinline__ double to_double(Pair p) { return (double)p.hi + (double)p.lo; }

__device__ __forceinline__ float ex2f(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float lg2f(float x) {
    float y;
    asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// log-sum-exp of the valid terms (hi[i] + lo[i]) + w[i]; kNeg when none is valid.
template <int N>
__device__ __forceinline__ Pair lse_pair(const float (&hi)[N], const float (&lo)[N], const float (&w)[N],
                                         const bool (&ok)[N]) {
    float lead[N];
#pragma unroll
    for (int i = 0; i < N; ++i) lead[i] = ok[i] ? hi[i] + w[i] : kNeg;
    float mx[N];
#pragma unroll
    for (int i = 0; i < N; ++i) mx[i] = lead[i];
#pragma unroll
    for (int s = 1; s < N; s *= 2)
#pragma unroll
        for (int i = 0; i + s < N; i += 2 * s) mx[i] = fmaxf(mx[i], mx[i + s]);
    const float m = mx[0];
    if (m <= 0.5f * kNeg) return {kNeg, 0.f};
    float e[N];
#pragma unroll
    for (int i = 0; i < N; ++i) e[i] = ok[i] ? ex2f((((hi[i] - m) + w[i]) + lo[i]) * kLog2e_f) : 0.f;
#pragma unroll
    for (int s = 1; s < N; s *= 2)
#pragma unroll
        for (int i = 0; i + s < N; i += 2 * s) e[i] += e[i + s];
    return two_sum(m, lg2f(e[0]) * kLn2_f);
}

struct LatArgs {
    LatticeMeta m;
    const float* lpb;  // diagonal-major weights (T_b x U_b grid per utterance)
    const float* lpy;
    const float* lpd;  // TDT: (nodes, n_dur); nullptr for RNN-T
    const int32_t* durations;
    int n_dur, has_zero;
    double* alpha;  // forward output / backward input; diagonal-major
    double* beta;   // backward: diagonal-major over the (T_b + 1)-row grid
    const float* grad_loss;
    float* cb;    // node-major: grad_loss * blank / token posteriors
    float* ct;
    float* gdur;  // node-major (nodes, n_dur): d loss / d duration logit (TDT)
    float* log_prob;
    float* loss;
    int ks;  // positions per thread
};

template <int N>
__device__ __forceinline__ void cp_async_wait_n() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Number of nodes on diagonal g of a rows x cols grid (0 outside it).
__device__ __forceinline__ int diag_len(int g, int rows, int cols) {
    const int lo = max(0, g - rows + 1), hi = min(g, cols - 1);
    return hi >= lo ? hi - lo + 1 : 0;
}

// Barrier over the CTA's active threads (a multiple of 32).
__device__ __forceinline__ void bar_active(int act) {
    if (act > 32)
        asm volatile("bar.sync 1, %0;" ::"r"(act) : "memory");
    else
        __syncwarp();
}

// Copies the weights of one diagonal (nodes n0 .. n0 + len - 1 of the
// diagonal-major arrays, label positions ulo ..) into a staging slot laid out
// by label position: lpb [upos], lpy [upos], lpd [upos * n_dur]; for the
// backward also alpha (a0: the diagonal's first node in alpha's own grid).
template <bool TDT, bool ALPHA>
__device__ __forceinline__ void stage_diag(float* slot, double* aslot, int upos, const LatArgs& a, int n0, int ulo,
                                           int len, const double* a0, int tid, int nt) {
    for (int i = tid; i < len; i += nt) {
        cp_async4(slot + ulo + i, a.lpb + n0 + i);
        cp_async4(slot + upos + ulo + i, a.lpy + n0 + i);
        if (ALPHA) cp_async8(aslot + ulo + i, a0 + i);
    }
    if (TDT) {
        const int nd = a.n_dur;
        const float* src = a.lpd + (int64_t)n0 * nd;
        float* dst = slot + 2 * upos + ulo * nd;
        for (int i = tid; i < len * nd; i += nt) cp_async4(dst + i, src + i);
    }
}

// Log-probability of the duration classes of value dv at one node (ld: its
// n_dur class log-probs): a direct read when classes are unique (k: the class
// of dv, clamped to 0 when there is none: the term is then invalid anyway).
template <int MAXD>
__device__ __forceinline__ float dur_lp(bool uniq, const int (&k)[MAXD + 1], const DurTable<MAXD>& dt,
                                        const float* ld, int dv, uint32_t mask) {
    if (uniq) return ld[k[dv]];
    return dur_weight(ld, 1, mask, dt.single[dv]);
}

// ------------------------------------------------------------------ forward

template <bool RNNT, int MAXD, bool GM>
__global__ void __launch_bounds__(kMaxThreads) lattice_alpha_kernel(LatArgs a) {
    constexpr bool TDT = !RNNT;
    constexpr int RV = MAXD + 2;           // recursion variable of diagonals g - MAXD - 1 .. g
    constexpr int S = MAXD + kAhead + 1;   // weight diagonals g - MAXD - 1 .. g + P - 1
    constexpr int NB = RNNT ? 1 : MAXD;    // blank durations 1 .. NB
    constexpr int NTK = RNNT ? 1 : MAXD + 1;  // token durations 0 .. NTK - 1
    constexpr int N = NB + NTK + 1;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int nt = blockDim.x, ks = a.ks, upos = nt * ks;
    const int b = blockIdx.x;
    const int Tb = a.m.Tb[b], Ub = a.m.Ub[b], off = a.m.off[b];
    // one position per thread: only the warps holding positions < U_b take part
    const int act = ks == 1 ? min(nt, (Ub + 31) & ~31) : nt;
    const int tid = threadIdx.x;
    if (tid >= act) return;
    const int arows = RNNT ? Tb : Tb + 1;  // rows of the stored alpha grid
    const int xoff = RNNT ? off : a.m.aoff[b];
    const int nd = TDT ? a.n_dur : 0;
    const DurTable<MAXD> dt = make_dur_table<MAXD>(TDT ? a.durations : nullptr, nd, a.has_zero);
    const bool uniq = TDT ? dt.uniq : true;
    int kc[MAXD + 1];
    bool hb[MAXD + 1], ht[MAXD + 1];
    uint32_t mk[MAXD + 1];
#pragma unroll
    for (int d = 0; d <= MAXD; ++d) {
        kc[d] = TDT ? max(d == 0 ? dt.tok0_k : dt.single[d], 0) : 0;
        mk[d] = TDT ? (d == 0 ? dt.tok0 : dt.mask[d]) : 0u;
        hb[d] = RNNT ? d == 1 : (d >= 1 && dt.mask[d] != 0u);
        ht[d] = RNNT ? d == 0 : mk[d] != 0u;
    }

    Pair* ring = reinterpret_cast<Pair*>(smem_raw);
    float* stg = reinterpret_cast<float*>(ring + (GM ? 0 : RV * upos));
    const int slot_floats = upos * (2 + nd);
    // staging of weight diagonal w: its first node and first label position, tracked incrementally
    int wn = 0, wlo = 0;
    if (!GM) {
        for (int i = tid; i < RV * upos; i += act) ring[i] = {kNeg, 0.f};
        cp_async_commit();  // weight diagonal -1: nothing
        for (int w = 0; w < kAhead - 1; ++w) {
            const int len = diag_len(w, Tb, Ub);
            if (len > 0) stage_diag<TDT, false>(stg + (w % S) * slot_floats, nullptr, upos, a, off + wn, wlo, len,
                                                nullptr, tid, act);
            cp_async_commit();
            wn += len;
            wlo = max(0, w + 1 - Tb + 1);
        }
    }
    int an = 0;  // first node of diagonal g in alpha's grid
    int sg = 0, rg = 0;  // g % S, g % RV
    const int last = Tb + Ub - 1;  // last diagonal of the (T_b + 1)-row grid
    for (int g = 0; g <= last; ++g) {
        if (!GM) cp_async_wait_n<kAhead - 1>();  // weight diagonal g - 1 landed (this thread's copies)
        bar_active(act);  // ... for every thread; diagonal g - 1 of the recursion visible
        if (!GM) {
            // weight diagonal g + P - 1 into the slot of g - MAXD - 2, which no thread reads any more
            const int w = g + kAhead - 1;
            const int len = diag_len(w, Tb, Ub);
            int k = sg + kAhead - 1;
            k -= k >= S ? S : 0;
            if (len > 0) stage_diag<TDT, false>(stg + k * slot_floats, nullptr, upos, a, off + wn, wlo, len, nullptr,
                                                tid, act);
            cp_async_commit();
            wn += len;
            wlo = max(0, w + 1 - Tb + 1);
        }
        // sources on diagonal g - s, s = 1 .. MAXD + 1
        const float* ws[MAXD + 2];
        const Pair* rs[MAXD + 2];
#pragma unroll
        for (int s2 = 1; s2 <= MAXD + 1; ++s2) {
            int k = sg - s2;
            k += k < 0 ? S : 0;
            int r = rg - s2;
            r += r < 0 ? RV : 0;
            ws[s2] = stg + k * slot_floats;
            rs[s2] = ring + r * upos;
        }
        const int alo = max(0, g - arows + 1);
#pragma unroll 1
        for (int j = 0; j < ks; ++j) {
            const int u = j * nt + tid;
            const int t = g - u;
            const bool in = u < Ub && t >= 0 && t <= Tb;
            Pair x = {kNeg, 0.f};
            if (in) {
                const int ul = u >= 1 ? u - 1 : 0;
                float hi[N], lo[N], wv[N];
                bool ok[N];
#pragma unroll
                for (int d = 1; d <= NB; ++d) {  // blank (t - d, u) -> (t, u): diagonal g - d
                    Pair src;
                    float w;
                    if (GM) {
                        const int sc = max(t - d, 0);
                        src = to_pair(a.alpha[xoff + diag_index(sc, u, arows, Ub)]);
                        const int n = off + diag_index(sc, u, Tb, Ub);
                        w = __ldg(a.lpb + n) + (TDT ? dur_lp<MAXD>(uniq, kc, dt, a.lpd + (int64_t)n * nd, d, mk[d]) : 0.f);
                    } else {
                        src = rs[d][u];
                        w = ws[d][u] + (TDT ? dur_lp<MAXD>(uniq, kc, dt, ws[d] + 2 * upos + u * nd, d, mk[d]) : 0.f);
                    }
                    hi[d - 1] = src.hi;
                    lo[d - 1] = src.lo;
                    wv[d - 1] = w;
                    ok[d - 1] = hb[d] && t - d >= 0;
                }
#pragma unroll
                for (int k = 0; k < NTK; ++k) {  // token (t - d, u - 1) -> (t, u): diagonal g - d - 1
                    const int d = RNNT ? 0 : k;
                    Pair src;
                    float w;
                    if (GM) {
                        const int sc = min(max(t - d, 0), Tb - 1);
                        src = to_pair(a.alpha[xoff + diag_index(sc, ul, arows, Ub)]);
                        const int n = off + diag_index(sc, ul, Tb, Ub);
                        w = __ldg(a.lpy + n) + (TDT ? dur_lp<MAXD>(uniq, kc, dt, a.lpd + (int64_t)n * nd, d, mk[d]) : 0.f);
                    } else {
                        src = rs[d + 1][ul];
                        w = ws[d + 1][upos + ul] +
                            (TDT ? dur_lp<MAXD>(uniq, kc, dt, ws[d + 1] + 2 * upos + ul * nd, d, mk[d]) : 0.f);
                    }
                    hi[NB + k] = src.hi;
                    lo[NB + k] = src.lo;
                    wv[NB + k] = w;
                    ok[NB + k] = ht[d] && u >= 1 && t - d >= 0 && t - d < Tb;
                }
                hi[N - 1] = 0.f;  // the start node (0, 0)
                lo[N - 1] = 0.f;
                wv[N - 1] = 0.f;
                ok[N - 1] = t == 0 && u == 0;
                x = lse_pair(hi, lo, wv, ok);
                if (RNNT ? t < Tb : true) a.alpha[xoff + an + (u - alo)] = to_double(x);
                if (t == Tb && u == Ub - 1) {  // terminal (rnnt.cu:242-248, tdt.cu:291-295)
                    const double lp = to_double(x);
                    a.log_prob[b] = (float)lp;
                    a.loss[b] = (float)(-lp);
                }
            }
            if (!GM) ring[rg * upos + u] = x;  // slot of diagonal g - MAXD - 2: unused now
        }
        an += diag_len(g, arows, Ub);
        sg = sg + 1 == S ? 0 : sg + 1;
        rg = rg + 1 == RV ? 0 : rg + 1;
    }
    if (!GM) cp_async_wait_n<0>();
}

// ----------------------------------------------------------------- backward
//
// beta(T_b, u) is 0 at u = U_b - 1 and log zero elsewhere; for t < T_b the node
// also writes its posteriors: cb = grad_loss * sum of blank-edge posteriors,
// ct = grad_loss * sum of token-edge posteriors, and (TDT) the duration-logit
// gradient gl * (g_k - P_dur(k) * sum_k' g_k') with g_k = -(posteriors of the
// edges using class k) (tdt.cu:400-426 + 475-500). Posteriors cover every
// duration class, also zero-duration classes other than the d = 0 token
// chain's. log Z is the forward's terminal, recomputed in float64.

template <bool RNNT, int MAXD, bool GM>
__global__ void __launch_bounds__(kMaxThreads) lattice_beta_kernel(LatArgs a) {
    constexpr bool TDT = !RNNT;
    constexpr int RV = MAXD + 2;    // beta of diagonals g .. g + MAXD + 1
    constexpr int S = kAhead + 1;   // weight diagonals g - P .. g
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int nt = blockDim.x, ks = a.ks, upos = nt * ks;
    const int b = blockIdx.x;
    const int Tb = a.m.Tb[b], Ub = a.m.Ub[b], off = a.m.off[b], boff = a.m.aoff[b];
    const int act = ks == 1 ? min(nt, (Ub + 31) & ~31) : nt;
    const int tid = threadIdx.x;
    if (tid >= act) return;
    const int arows = RNNT ? Tb : Tb + 1;
    const int aoff = RNNT ? off : boff;
    const int nd = TDT ? a.n_dur : 0;
    const DurTable<MAXD> dt = make_dur_table<MAXD>(TDT ? a.durations : nullptr, nd, a.has_zero);
    const bool uniq = TDT ? dt.uniq : true;
    int kc[MAXD + 1];
    bool hb[MAXD + 1], ht[MAXD + 1];
    uint32_t mk[MAXD + 1];
#pragma unroll
    for (int d = 0; d <= MAXD; ++d) {
        kc[d] = TDT ? max(d == 0 ? dt.tok0_k : dt.single[d], 0) : 0;
        mk[d] = TDT ? (d == 0 ? dt.tok0 : dt.mask[d]) : 0u;
        hb[d] = RNNT ? d == 1 : (d >= 1 && dt.mask[d] != 0u);
        ht[d] = RNNT ? d == 0 : dt.mask[d] != 0u;  // posteriors: every class of value d
    }
    const bool chain0 = RNNT || dt.tok0 != 0u;  // the recursion's d = 0 token edge

    Pair* ring = reinterpret_cast<Pair*>(smem_raw);
    double* astg = reinterpret_cast<double*>(ring + (GM ? 0 : RV * upos));
    float* stg = reinterpret_cast<float*>(astg + (GM ? 0 : S * upos));
    const int slot_floats = upos * (2 + nd);
    // log Z in float64 from the forward variable
    const double logz = RNNT ? a.alpha[aoff + diag_index(Tb - 1, Ub - 1, Tb, Ub)] +
                                   (double)a.lpb[off + diag_index(Tb - 1, Ub - 1, Tb, Ub)]
                             : a.alpha[aoff + diag_index(Tb, Ub - 1, Tb + 1, Ub)];
    const float gl = a.grad_loss[b];
    const int first = Tb + Ub - 1;
    // staging walks weight diagonals downwards: wn = one past the last node of diagonal w
    int wn = Tb * Ub;
    if (!GM) {
        for (int i = tid; i < RV * upos; i += act) ring[i] = {kNeg, 0.f};
        for (int k = 0; k < kAhead; ++k) {
            const int w = first - k;  // the top diagonal (row T_b only) has no weights
            const int len = diag_len(w, Tb, Ub);
            if (len > 0) {
                wn -= len;
                const int ulo = max(0, w - Tb + 1);
                const double* a0 = a.alpha + aoff + diag_index(w - ulo, ulo, arows, Ub);
                stage_diag<TDT, true>(stg + (w % S) * slot_floats, astg + (w % S) * upos, upos, a, off + wn, ulo, len,
                                      a0, tid, act);
            }
            cp_async_commit();
        }
    }
    int bn = (Tb + 1) * Ub;  // one past diagonal g's last node in beta's grid
    for (int g = first; g >= 0; --g) {
        if (!GM) cp_async_wait_n<kAhead - 1>();  // weight diagonal g landed (this thread's copies)
        bar_active(act);  // ... for every thread; diagonal g + 1 of the recursion visible
        const int sg = g % S, rg = g % RV;
        if (!GM) {
            // weight diagonal g - P into the slot of g + 1, which no thread reads any more
            const int w = g - kAhead;
            const int len = w >= 0 ? diag_len(w, Tb, Ub) : 0;
            if (len > 0) {
                wn -= len;
                const int ulo = max(0, w - Tb + 1);
                const double* a0 = a.alpha + aoff + diag_index(w - ulo, ulo, arows, Ub);
                const int k = w % S;
                stage_diag<TDT, true>(stg + k * slot_floats, astg + k * upos, upos, a, off + wn, ulo, len, a0, tid,
                                      act);
            }
            cp_async_commit();
        }
        const Pair* rs[MAXD + 2];  // beta of diagonal g + s, s = 1 .. MAXD + 1
#pragma unroll
        for (int s2 = 1; s2 <= MAXD + 1; ++s2) {
            int r = rg + s2;
            r -= r >= RV ? RV : 0;
            rs[s2] = ring + r * upos;
        }
        const float* sl = stg + sg * slot_floats;
        const double* sa = astg + sg * upos;
        bn -= diag_len(g, Tb + 1, Ub);
        const int blo = max(0, g - Tb);
#pragma unroll 1
        for (int j = 0; j < ks; ++j) {
            const int u = j * nt + tid;
            const int t = g - u;
            const bool in = u < Ub && t >= 0 && t <= Tb;
            Pair x = {kNeg, 0.f};
            if (in && t == Tb) {
                x = {u == Ub - 1 ? 0.f : kNeg, 0.f};
            } else if (in) {
                const bool can_tok = u < Ub - 1;
                const int ur = can_tok ? u + 1 : u;
                float lb, ly;
                const float* ld = nullptr;
                double al;
                if (GM) {
                    const int n = off + diag_index(t, u, Tb, Ub);
                    lb = __ldg(a.lpb + n);
                    ly = __ldg(a.lpy + n);
                    if (TDT) ld = a.lpd + (int64_t)n * nd;
                    al = a.alpha[aoff + diag_index(t, u, arows, Ub)];
                } else {
                    lb = sl[u];
                    ly = sl[upos + u];
                    if (TDT) ld = sl + 2 * upos + u * nd;
                    al = sa[u];
                }
                // beta at the edges' destinations: blank (t + d, u), token (t + d, u + 1)
                Pair bd[MAXD + 1], td[MAXD + 1];
                bool vb[MAXD + 1], vt[MAXD + 1];
#pragma unroll
                for (int d = 0; d <= MAXD; ++d) {
                    vb[d] = hb[d] && t + d <= Tb;
                    vt[d] = ht[d] && can_tok && t + d <= Tb;
                    if (GM) {
                        const int tc = min(t + d, Tb);
                        bd[d] = to_pair(a.beta[boff + diag_index(tc, u, Tb + 1, Ub)]);
                        td[d] = to_pair(a.beta[boff + diag_index(tc, ur, Tb + 1, Ub)]);
                    } else {
                        bd[d] = d >= 1 ? rs[d][u] : Pair{kNeg, 0.f};
                        td[d] = rs[d + 1][ur];
                    }
                }
                // recursion: duration weight per value d (log-summed over its classes;
                // the d = 0 token chain uses the first zero-duration class only)
                float ldv[MAXD + 1];
#pragma unroll
                for (int d = 0; d <= MAXD; ++d) ldv[d] = TDT ? dur_lp<MAXD>(uniq, kc, dt, ld, d, mk[d]) : 0.f;
                constexpr int N = 2 * (MAXD + 1);
                float hi[N], lo[N], wv[N];
                bool ok[N];
#pragma unroll
                for (int d = 0; d <= MAXD; ++d) {
                    hi[d] = bd[d].hi;
                    lo[d] = bd[d].lo;
                    wv[d] = lb + ldv[d];
                    ok[d] = vb[d];
                    hi[MAXD + 1 + d] = td[d].hi;
                    lo[MAXD + 1 + d] = td[d].lo;
                    wv[MAXD + 1 + d] = ly + ldv[d];
                    ok[MAXD + 1 + d] = vt[d] && (d > 0 || chain0);
                }
                x = lse_pair(hi, lo, wv, ok);

                // edge posteriors exp(alpha + w + beta(dst) - log Z); alpha - log Z as
                // an exact pair, so that adding beta (about minus it) cancels exactly
                const Pair az = to_pair(al - logz);
                float eb[MAXD + 1], et[MAXD + 1];  // exponents without the duration weight
#pragma unroll
                for (int d = 0; d <= MAXD; ++d) {
                    eb[d] = vb[d] ? ((az.hi + bd[d].hi) + (az.lo + bd[d].lo)) + lb : -INFINITY;
                    et[d] = vt[d] ? ((az.hi + td[d].hi) + (az.lo + td[d].lo)) + ly : -INFINITY;
                }
                float bp = 0.f, tp = 0.f;
                const int nn = off + t * Ub + u;  // node-major: the backward joint reads these
                if (RNNT) {
                    bp = ex2f(eb[1] * kLog2e_f);
                    tp = ex2f(et[0] * kLog2e_f);
                } else if (uniq) {
                    float gk[MAXD + 1], gsum = 0.f;
#pragma unroll
                    for (int d = 0; d <= MAXD; ++d) {
                        const float gb = ex2f((eb[d] + ldv[d]) * kLog2e_f);
                        const float gt = ex2f((et[d] + ldv[d]) * kLog2e_f);
                        bp += gb;
                        tp += gt;
                        gk[d] = -(gb + gt);
                        gsum += gk[d];
                    }
                    float* gd = a.gdur + (int64_t)nn * nd;
#pragma unroll
                    for (int d = 0; d <= MAXD; ++d)
                        if (dt.single[d] >= 0) gd[dt.single[d]] = gl * (gk[d] - ex2f(ldv[d] * kLog2e_f) * gsum);
                } else {
                    // several classes share a duration value: every class's edges,
                    // each with its own class log-prob
                    float gi[kTdtMaxDurClasses];
                    float gsum = 0.f;
                    for (int k = 0; k < nd; ++k) {
                        const int dv = a.durations[k];
                        float g2 = 0.f;
                        if (dv >= 0 && dv <= MAXD) {
                            const float lk = ld[k];
                            const float gb = ex2f((eb[dv] + lk) * kLog2e_f);
                            const float gt = ex2f((et[dv] + lk) * kLog2e_f);
                            bp += gb;
                            tp += gt;
                            g2 = -(gb + gt);
                        }
                        gi[k] = g2;
                        gsum += g2;
                    }
                    float* gd = a.gdur + (int64_t)nn * nd;
                    for (int k = 0; k < nd; ++k) gd[k] = gl * (gi[k] - ex2f(ld[k] * kLog2e_f) * gsum);
                }
                a.cb[nn] = gl * bp;
                a.ct[nn] = gl * tp;
            }
            if (in && (GM || TDT)) a.beta[boff + bn + (u - blo)] = to_double(x);
            if (!GM) ring[rg * upos + u] = x;  // slot of diagonal g + MAXD + 2: unused now
        }
    }
    if (!GM) cp_async_wait_n<0>();
}

// ------------------------------------------------------------------ launchers

size_t alpha_smem(bool gm, int maxd, int n_dur, int upos) {
    if (gm) return 0;
    return sizeof(Pair) * (size_t)(maxd + 2) * upos + sizeof(float) * (size_t)(maxd + kAhead + 1) * upos * (2 + n_dur);
}

size_t beta_smem(bool gm, int maxd, int n_dur, int upos) {
    if (gm) return 0;
    const int S = kAhead + 1;
    return sizeof(Pair) * (size_t)(maxd + 2) * upos + sizeof(double) * (size_t)S * upos +
           sizeof(float) * (size_t)S * upos * (2 + n_dur);
}

constexpr size_t kSmemLimit = 200 * 1024;

template <typename Kern>
int prepare(Kern k, size_t smem, int threads) {
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return ASR_ERR_UNSUPPORTED;
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, k) != cudaSuccess || threads > fa.maxThreadsPerBlock) return ASR_ERR_UNSUPPORTED;
    return ASR_OK;
}

template <bool FWD, bool RNNT, int MAXD>
int launch_lattice(LatArgs a, int B, int U, const char* name, cudaStream_t st) {
    if (U < 1 || U > kMaxLabelPositions) return ASR_ERR_UNSUPPORTED;
    const int nt = std::min(kMaxThreads, (U + 31) / 32 * 32);
    a.ks = (U + nt - 1) / nt;
    const int upos = nt * a.ks;
    const int nd = RNNT ? 0 : a.n_dur;
    size_t smem = FWD ? alpha_smem(false, MAXD, nd, upos) : beta_smem(false, MAXD, nd, upos);
    const bool gm = smem > kSmemLimit;
    if (gm) {
        if (!FWD && !a.beta) return ASR_ERR_UNSUPPORTED;
        smem = 0;
    }
    auto k = FWD ? (gm ? lattice_alpha_kernel<RNNT, MAXD, true> : lattice_alpha_kernel<RNNT, MAXD, false>)
                 : (gm ? lattice_beta_kernel<RNNT, MAXD, true> : lattice_beta_kernel<RNNT, MAXD, false>);
    if (int rc = prepare(k, smem, nt)) return rc;
    KernelTimer kt(name, st);
    k<<<B, nt, smem, st>>>(a);
    ASR_LAUNCH_CHECK();
    return ASR_OK;
}

int tdt_maxd(int max_duration) {
    if (max_duration <= 2) return 2;
    if (max_duration <= 4) return 4;
    if (max_duration <= 8) return 8;
    if (max_duration <= 16) return 16;
    return 0;
}

template <bool FWD>
int launch_tdt(const LatArgs& a, int B, int U, int max_duration, const char* name, cudaStream_t st) {
    if (a.n_dur < 1 || a.n_dur > kTdtMaxDurClasses) return ASR_ERR_UNSUPPORTED;
    switch (tdt_maxd(max_duration)) {
        case 2: return launch_lattice<FWD, false, 2>(a, B, U, name, st);
        case 4: return launch_lattice<FWD, false, 4>(a, B, U, name, st);
        case 8: return launch_lattice<FWD, false, 8>(a, B, U, name, st);
        case 16: return launch_lattice<FWD, false, 16>(a, B, U, name, st);
        default: return ASR_ERR_UNSUPPORTED;
    }
}

}  // namespace

int launch_rnnt_alpha(const LatticeMeta& m, int B, int U, const float* lpb, const float* lpy, double* alpha,
                      float* log_prob, float* loss, cudaStream_t st) {
    LatArgs a{};
    a.m = m;
    a.lpb = lpb;
    a.lpy = lpy;
    a.alpha = alpha;
    a.log_prob = log_prob;
    a.loss = loss;
    return launch_lattice<true, true, 1>(a, B, U, "rnnt_alpha", st);
}

int launch_rnnt_beta(const LatticeMeta& m, int B, int U, const float* lpb, const float* lpy, const double* alpha,
                     const float* grad_loss, float* cb, float* ct, double* beta, cudaStream_t st) {
    LatArgs a{};
    a.m = m;
    a.lpb = lpb;
    a.lpy = lpy;
    a.alpha = const_cast<double*>(alpha);
    a.beta = beta;
    a.grad_loss = grad_loss;
    a.cb = cb;
    a.ct = ct;
    return launch_lattice<false, true, 1>(a, B, U, "rnnt_beta_posteriors", st);
}

int launch_tdt_alpha(const LatticeMeta& m, int B, int U, int max_duration, const int32_t* durations, int n_dur,
                     int has_zero, const float* lpb, const float* lpy, const float* lpd, double* alpha,
                     float* log_prob, float* loss, cudaStream_t st) {
    LatArgs a{};
    a.m = m;
    a.lpb = lpb;
    a.lpy = lpy;
    a.lpd = lpd;
    a.durations = durations;
    a.n_dur = n_dur;
    a.has_zero = has_zero;
    a.alpha = alpha;
    a.log_prob = log_prob;
    a.loss = loss;
    return launch_tdt<true>(a, B, U, max_duration, "tdt_alpha", st);
}

int launch_tdt_beta(const LatticeMeta& m, int B, int U, int max_duration, const int32_t* durations, int n_dur,
                    int has_zero, const float* lpb, const float* lpy, const float* lpd, const double* alpha,
                    const float* grad_loss, float* cb, float* ct, float* gdur, double* beta, cudaStream_t st) {
    LatArgs a{};
    a.m = m;
    a.lpb = lpb;
    a.lpy = lpy;
    a.lpd = lpd;
    a.durations = durations;
    a.n_dur = n_dur;
    a.has_zero = has_zero;
    a.alpha = const_cast<double*>(alpha);
    a.beta = beta;
    a.grad_loss = grad_loss;
    a.cb = cb;
    a.ct = ct;
    a.gdur = gdur;
    return launch_tdt<false>(a, B, U, max_duration, "tdt_beta_posteriors", st);
}

}  // namespace asr
