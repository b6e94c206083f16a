// RNN-T lattice recursions: alpha (forward) and beta fused with the edge
// posteriors (backward). Reference semantics: rnnt.cu:218-317.
//
// One CTA per utterance sweeps anti-diagonals g = t + u with one thread per
// label position u. Every node on a diagonal depends only on the previous
// diagonal: (t-1, u) through the blank edge and (t, u-1) through the label edge.
// The outgoing values alpha + log_P (forward) or the recursion variable
// (backward) of the last two diagonals sit in a float64 shared-memory ring, so a
// thread reads its neighbour position directly and one __syncthreads separates
// consecutive diagonals (a diagonal writes the slot that the diagonal before
// the previous one used, which no thread reads any more). Each thread copies its
// next node's edge log-probs (and alpha, backward) into shared memory with
// cp.async one diagonal ahead.
#include <algorithm>

#include "dp.cuh"

namespace asr {
namespace {

// cp.async copies of node n's blank / label log-probs into slot `slot` of the
// two-diagonal weight ring [slot][2][NT] (own column only).
__device__ __forceinline__ void prefetch_edge(float* wring, int slot, int NT, int u, int n, const float* lpb,
                                              const float* lpy) {
    float* dst = wring + slot * 2 * NT + u;
    cp_async4(dst, lpb + n);
    cp_async4(dst + NT, lpy + n);
}

// Shared memory: vring[2][2][NT] doubles (recursion values of the two most recent
// diagonals), wring[2][2][NT] floats, aring[2][NT] doubles (backward).
size_t rnnt_smem(int NT, bool bwd) {
    return sizeof(double) * 4 * (size_t)NT + sizeof(float) * 4 * (size_t)NT + (bwd ? sizeof(double) * 2 * NT : 0);
}

__global__ void rnnt_alpha_kernel(LatticeMeta m, int NT, const float* __restrict__ lpb, const float* __restrict__ lpy,
                                  double* __restrict__ alpha, float* __restrict__ log_prob, float* __restrict__ loss) {
    extern __shared__ __align__(16) unsigned char dp_raw[];
    double* hring = reinterpret_cast<double*>(dp_raw);        // [slot][blank-out, label-out][NT]
    float* wring = reinterpret_cast<float*>(hring + 4 * NT);  // [slot][blank, label][NT]
    const int u = threadIdx.x, b = blockIdx.x;
    const int Tb = m.Tb[b], Ub = m.Ub[b], off = m.off[b];
    const bool lane_in = u < Ub;
    for (int i = u; i < 4 * NT; i += NT) hring[i] = kNeg;
    if (u == 0) prefetch_edge(wring, 0, NT, 0, off, lpb, lpy);
    cp_async_commit();
    const int last = Tb + Ub - 2;
    for (int g = 0; g <= last; ++g) {
        {
            const int t1 = g + 1 - u;
            if (g < last && lane_in && t1 >= 0 && t1 < Tb)
                prefetch_edge(wring, (g + 1) & 1, NT, u, off + t1 * Ub + u, lpb, lpy);
            cp_async_commit();
        }
        cp_async_wait_prev();
        __syncthreads();  // edge weights of diagonal g and outgoing values of diagonal g - 1 visible
        const int t = g - u;
        const int prev = (g + 1) & 1;  // slot of diagonal g - 1
        double hb = kNeg, hy = kNeg;
        if (lane_in && t >= 0 && t < Tb) {
            // blank from (t-1, u): same column; label from (t, u-1): left column
            const double from_blank = t > 0 ? hring[(prev * 2 + 0) * NT + u] : (double)kNeg;
            const double from_label = u > 0 ? hring[(prev * 2 + 1) * NT + u - 1] : (double)kNeg;
            const double a = (t == 0 && u == 0) ? 0.0 : lae_d(from_blank, from_label);
            const int n = off + t * Ub + u;
            const float* w = wring + (g & 1) * 2 * NT + u;
            const float lb = w[0], ly = w[NT];
            alpha[n] = a;
            hb = a + lb;
            hy = a + ly;
            if (t == Tb - 1 && u == Ub - 1) {  // terminal blank (rnnt.cu:242-248)
                log_prob[b] = (float)(a + lb);
                loss[b] = (float)(-(a + lb));
            }
        }
        hring[((g & 1) * 2 + 0) * NT + u] = hb;
        hring[((g & 1) * 2 + 1) * NT + u] = hy;
    }
}

// Writes cb = grad_loss * blank posterior and ct = grad_loss * label posterior per
// node. log P(y|x) is recomputed from the float64 forward variable.
__global__ void rnnt_beta_kernel(LatticeMeta m, int NT, const float* __restrict__ lpb, const float* __restrict__ lpy,
                                 const double* __restrict__ alpha, const float* __restrict__ grad_loss,
                                 float* __restrict__ cb, float* __restrict__ ct) {
    extern __shared__ __align__(16) unsigned char dp_raw[];
    double* bring = reinterpret_cast<double*>(dp_raw);             // [slot][NT] (2 of the 4*NT doubles used)
    float* wring = reinterpret_cast<float*>(bring + 4 * NT);       // [slot][blank, label][NT]
    double* aring = reinterpret_cast<double*>(wring + 4 * NT);     // [slot][NT]
    const int u = threadIdx.x, b = blockIdx.x;
    const int Tb = m.Tb[b], Ub = m.Ub[b], off = m.off[b];
    const bool lane_in = u < Ub;
    const int nterm = off + (Tb - 1) * Ub + Ub - 1;
    const double logZ = alpha[nterm] + lpb[nterm];
    const float gl = grad_loss[b];
    for (int i = u; i < 4 * NT; i += NT) bring[i] = kNeg;
    auto prefetch = [&](int g) {
        const int t = g - u;
        if (g >= 0 && lane_in && t >= 0 && t < Tb) {
            const int n = off + t * Ub + u;
            prefetch_edge(wring, g & 1, NT, u, n, lpb, lpy);
            cp_async8(aring + (g & 1) * NT + u, alpha + n);
        }
        cp_async_commit();
    };
    const int first = Tb + Ub - 2;
    prefetch(first);
    for (int g = first; g >= 0; --g) {
        prefetch(g - 1);
        cp_async_wait_prev();
        __syncthreads();  // weights of diagonal g and beta of diagonal g + 1 visible
        const int t = g - u;
        const int nxt = (g + 1) & 1;  // slot of diagonal g + 1
        double be = kNeg;
        if (lane_in && t >= 0 && t < Tb) {
            const int n = off + t * Ub + u;
            const float* w = wring + (g & 1) * 2 * NT + u;
            const float lb = w[0], ly = w[NT];
            const double a = aring[(g & 1) * NT + u];
            const double b_t1 = bring[nxt * NT + u];                                    // beta(t+1, u)
            const double b_u1 = u + 1 < NT ? bring[nxt * NT + u + 1] : (double)kNeg;  // beta(t, u+1)
            const bool term = (t == Tb - 1) && (u == Ub - 1);
            const bool can_blank = t < Tb - 1, can_label = u < Ub - 1;
            const double blank_term = term ? (double)lb : (can_blank ? lb + b_t1 : (double)kNeg);
            const double label_term = can_label ? ly + b_u1 : (double)kNeg;
            be = lae_d(blank_term, label_term);
            const float bp = term ? __expf((float)(a + lb - logZ))
                                  : (can_blank ? __expf((float)(a + lb + b_t1 - logZ)) : 0.f);
            const float tp = can_label ? __expf((float)(a + ly + b_u1 - logZ)) : 0.f;
            cb[n] = gl * bp;
            ct[n] = gl * tp;
        }
        bring[(g & 1) * NT + u] = be;
    }
}

int rnnt_threads(int U) { return (U + 31) / 32 * 32; }

template <typename Kern>
int set_smem(Kern k, size_t bytes) {
    if (bytes > 227 * 1024) return ASR_ERR_UNSUPPORTED;
    if (bytes > 48 * 1024 &&
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) != cudaSuccess)
        return ASR_ERR_UNSUPPORTED;
    return ASR_OK;
}

}  // namespace

int launch_rnnt_alpha(const LatticeMeta& m, int B, int U, const float* lpb, const float* lpy, double* alpha,
                      float* log_prob, float* loss, cudaStream_t st) {
    if (U > 1024) return ASR_ERR_UNSUPPORTED;
    const int NT = rnnt_threads(U);
    const size_t smem = rnnt_smem(NT, false);
    if (set_smem(rnnt_alpha_kernel, smem)) return ASR_ERR_UNSUPPORTED;
    KernelTimer kt("rnnt_alpha", st);
    rnnt_alpha_kernel<<<B, NT, smem, st>>>(m, NT, lpb, lpy, alpha, log_prob, loss);
    ASR_LAUNCH_CHECK();
    return ASR_OK;
}

int launch_rnnt_beta(const LatticeMeta& m, int B, int U, const float* lpb, const float* lpy, const double* alpha,
                     const float* grad_loss, float* cb, float* ct, cudaStream_t st) {
    if (U > 1024) return ASR_ERR_UNSUPPORTED;
    const int NT = rnnt_threads(U);
    const size_t smem = rnnt_smem(NT, true);
    if (set_smem(rnnt_beta_kernel, smem)) return ASR_ERR_UNSUPPORTED;
    KernelTimer kt("rnnt_beta_posteriors", st);
    rnnt_beta_kernel<<<B, NT, smem, st>>>(m, NT, lpb, lpy, alpha, grad_loss, cb, ct);
    ASR_LAUNCH_CHECK();
    return ASR_OK;
}

}  // namespace asr
