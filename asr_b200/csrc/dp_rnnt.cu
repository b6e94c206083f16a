// RNN-T lattice recursions: alpha (forward) and beta fused with the edge
// posteriors (backward). Reference semantics: rnnt.cu:218-317.
//
// One warp per utterance sweeps anti-diagonals g = t + u. Lane l owns the K
// consecutive label positions u = l*K .. l*K+K-1 in registers. Every node on a
// diagonal depends only on the previous diagonal: (t-1, u) is the same register
// one step earlier and (t, u-1) is the left register, or the left lane's last
// register for the block head (one shuffle per diagonal). The warp never
// synchronises with other warps, so T_b + U_b - 1 short steps bound the latency
// and many utterances run concurrently on every SM. The next diagonal's edge
// log-probs (and alpha, backward) are prefetched into shared memory with
// cp.async while the current one computes.
#include "dp.cuh"

namespace asr {
namespace {

// Utterances (warps) per block: fewer for wide label blocks so the static
// prefetch buffers stay under 48 KB.
template <int K>
constexpr int warps_per_block() {
    return K >= 16 ? 1 : (K >= 8 ? 2 : 4);
}

// Next-diagonal prefetch: [slot][j][{blank, label}][lane] floats, plus alpha
// (backward) as [slot][j][lane] doubles.
template <int K>
__device__ __forceinline__ void rnnt_prefetch(float* wb, double* ab, int g, int lane, int Tb, int Ub, int off,
                                              const float* lpb, const float* lpy, const double* alpha) {
    const int slot = g & 1;
#pragma unroll
    for (int j = 0; j < K; ++j) {
        const int u = lane * K + j, t = g - u;
        if (u < Ub && t >= 0 && t < Tb) {
            const int n = off + t * Ub + u;
            float* dst = wb + ((slot * K + j) * 2) * 32 + lane;
            cp_async4(dst, lpb + n);
            cp_async4(dst + 32, lpy + n);
            if (ab) cp_async8(ab + (slot * K + j) * 32 + lane, alpha + n);
        }
    }
    cp_async_commit();
}

template <int K>
__global__ void __launch_bounds__(32 * warps_per_block<K>())
    rnnt_alpha_kernel(LatticeMeta m, int B, const float* __restrict__ lpb, const float* __restrict__ lpy,
                      double* __restrict__ alpha, float* __restrict__ log_prob, float* __restrict__ loss) {
    __shared__ float wbuf_all[warps_per_block<K>()][2 * K * 2 * 32];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int b = blockIdx.x * warps_per_block<K>() + warp;
    if (b >= B) return;
    float* wb = wbuf_all[warp];
    const int Tb = m.Tb[b], Ub = m.Ub[b], off = m.off[b];
    // hb / hy: alpha + edge log-prob of the node this register held on the previous
    // diagonal (outgoing blank / label value), kNeg when that node was not in the lattice.
    double hb[K], hy[K];
#pragma unroll
    for (int j = 0; j < K; ++j) hb[j] = hy[j] = kNeg;
    const int last = Tb + Ub - 2;
    rnnt_prefetch<K>(wb, nullptr, 0, lane, Tb, Ub, off, lpb, lpy, nullptr);
    for (int g = 0; g <= last; ++g) {
        if (g < last)
            rnnt_prefetch<K>(wb, nullptr, g + 1, lane, Tb, Ub, off, lpb, lpy, nullptr);
        else
            cp_async_commit();
        cp_async_wait_prev();
        __syncwarp();
        double left = __shfl_up_sync(0xffffffffu, hy[K - 1], 1);
        if (lane == 0) left = kNeg;
        double nb[K], ny[K];
#pragma unroll
        for (int j = 0; j < K; ++j) {
            const int u = lane * K + j, t = g - u;
            nb[j] = ny[j] = kNeg;
            if (u < Ub && t >= 0 && t < Tb) {
                const double from_label = (j > 0) ? hy[j > 0 ? j - 1 : 0] : left;
                const double a = (t == 0 && u == 0) ? 0.0 : lae_d(hb[j], from_label);
                const int n = off + t * Ub + u;
                const float* w = wb + (((g & 1) * K + j) * 2) * 32 + lane;
                const float lb = w[0], ly = w[32];
                alpha[n] = a;
                nb[j] = a + lb;
                ny[j] = a + ly;
                if (t == Tb - 1 && u == Ub - 1) {  // terminal blank (rnnt.cu:242-248)
                    log_prob[b] = (float)(a + lb);
                    loss[b] = (float)(-(a + lb));
                }
            }
        }
        __syncwarp();
#pragma unroll
        for (int j = 0; j < K; ++j) {
            hb[j] = nb[j];
            hy[j] = ny[j];
        }
    }
}

// Writes cb = grad_loss * blank posterior and ct = grad_loss * label posterior per
// node. log P(y|x) is recomputed from the float64 forward variable.
template <int K>
__global__ void __launch_bounds__(32 * warps_per_block<K>())
    rnnt_beta_kernel(LatticeMeta m, int B, const float* __restrict__ lpb, const float* __restrict__ lpy,
                     const double* __restrict__ alpha, const float* __restrict__ grad_loss, float* __restrict__ cb,
                     float* __restrict__ ct) {
    __shared__ float wbuf_all[warps_per_block<K>()][2 * K * 2 * 32];
    __shared__ double abuf_all[warps_per_block<K>()][2 * K * 32];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int b = blockIdx.x * warps_per_block<K>() + warp;
    if (b >= B) return;
    float* wb = wbuf_all[warp];
    double* ab = abuf_all[warp];
    const int Tb = m.Tb[b], Ub = m.Ub[b], off = m.off[b];
    const int nterm = off + (Tb - 1) * Ub + Ub - 1;
    const double logZ = alpha[nterm] + lpb[nterm];
    const float gl = grad_loss[b];
    double bn[K];  // beta of the node this register held on diagonal g+1, i.e. (t+1, u)
#pragma unroll
    for (int j = 0; j < K; ++j) bn[j] = kNeg;
    const int first = Tb + Ub - 2;
    rnnt_prefetch<K>(wb, ab, first, lane, Tb, Ub, off, lpb, lpy, alpha);
    for (int g = first; g >= 0; --g) {
        if (g > 0)
            rnnt_prefetch<K>(wb, ab, g - 1, lane, Tb, Ub, off, lpb, lpy, alpha);
        else
            cp_async_commit();
        cp_async_wait_prev();
        __syncwarp();
        double right = __shfl_down_sync(0xffffffffu, bn[0], 1);  // (t, u+1) for the block tail
        if (lane == 31) right = kNeg;
        double nbeta[K];
#pragma unroll
        for (int j = 0; j < K; ++j) {
            const int u = lane * K + j, t = g - u;
            nbeta[j] = kNeg;
            if (u < Ub && t >= 0 && t < Tb) {
                const int n = off + t * Ub + u;
                const float* w = wb + (((g & 1) * K + j) * 2) * 32 + lane;
                const float lb = w[0], ly = w[32];
                const double a = ab[((g & 1) * K + j) * 32 + lane];
                const double b_t1 = bn[j];
                const double b_u1 = (j + 1 < K) ? bn[j + 1 < K ? j + 1 : 0] : right;
                const bool term = (t == Tb - 1) && (u == Ub - 1);
                const bool can_blank = t < Tb - 1, can_label = u < Ub - 1;
                const double blank_term = term ? (double)lb : (can_blank ? lb + b_t1 : (double)kNeg);
                const double label_term = can_label ? ly + b_u1 : (double)kNeg;
                nbeta[j] = lae_d(blank_term, label_term);
                const float bp = term ? __expf((float)(a + lb - logZ))
                                      : (can_blank ? __expf((float)(a + lb + b_t1 - logZ)) : 0.f);
                const float tp = can_label ? __expf((float)(a + ly + b_u1 - logZ)) : 0.f;
                cb[n] = gl * bp;
                ct[n] = gl * tp;
            }
        }
        __syncwarp();
#pragma unroll
        for (int j = 0; j < K; ++j) bn[j] = nbeta[j];
    }
}

template <int K>
int launch_rnnt_alpha_k(const LatticeMeta& m, int B, const float* lpb, const float* lpy, double* alpha, float* lp,
                        float* loss, cudaStream_t st) {
    KernelTimer kt("rnnt_alpha", st);
    rnnt_alpha_kernel<K><<<(B + warps_per_block<K>() - 1) / warps_per_block<K>(), 32 * warps_per_block<K>(), 0, st>>>(m, B, lpb, lpy, alpha, lp, loss);
    ASR_LAUNCH_CHECK();
    return ASR_OK;
}

template <int K>
int launch_rnnt_beta_k(const LatticeMeta& m, int B, const float* lpb, const float* lpy, const double* alpha,
                       const float* gl, float* cb, float* ct, cudaStream_t st) {
    KernelTimer kt("rnnt_beta_posteriors", st);
    rnnt_beta_kernel<K><<<(B + warps_per_block<K>() - 1) / warps_per_block<K>(), 32 * warps_per_block<K>(), 0, st>>>(m, B, lpb, lpy, alpha, gl, cb, ct);
    ASR_LAUNCH_CHECK();
    return ASR_OK;
}

}  // namespace

int launch_rnnt_alpha(const LatticeMeta& m, int B, int U, const float* lpb, const float* lpy, double* alpha,
                      float* log_prob, float* loss, cudaStream_t st) {
    switch (dp_lanes_k(U)) {
        case 1: return launch_rnnt_alpha_k<1>(m, B, lpb, lpy, alpha, log_prob, loss, st);
        case 2: return launch_rnnt_alpha_k<2>(m, B, lpb, lpy, alpha, log_prob, loss, st);
        case 4: return launch_rnnt_alpha_k<4>(m, B, lpb, lpy, alpha, log_prob, loss, st);
        case 8: return launch_rnnt_alpha_k<8>(m, B, lpb, lpy, alpha, log_prob, loss, st);
        case 16: return launch_rnnt_alpha_k<16>(m, B, lpb, lpy, alpha, log_prob, loss, st);
        default: return ASR_ERR_UNSUPPORTED;
    }
}

int launch_rnnt_beta(const LatticeMeta& m, int B, int U, const float* lpb, const float* lpy, const double* alpha,
                     const float* grad_loss, float* cb, float* ct, cudaStream_t st) {
    switch (dp_lanes_k(U)) {
        case 1: return launch_rnnt_beta_k<1>(m, B, lpb, lpy, alpha, grad_loss, cb, ct, st);
        case 2: return launch_rnnt_beta_k<2>(m, B, lpb, lpy, alpha, grad_loss, cb, ct, st);
        case 4: return launch_rnnt_beta_k<4>(m, B, lpb, lpy, alpha, grad_loss, cb, ct, st);
        case 8: return launch_rnnt_beta_k<8>(m, B, lpb, lpy, alpha, grad_loss, cb, ct, st);
        case 16: return launch_rnnt_beta_k<16>(m, B, lpb, lpy, alpha, grad_loss, cb, ct, st);
        default: return ASR_ERR_UNSUPPORTED;
    }
}

}  // namespace asr
