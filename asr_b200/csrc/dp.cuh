// Launchers of the lattice recursions (dp_rnnt.cu, dp_tdt.cu).
#pragma once

#include "common.cuh"

namespace asr {

// Largest label axis (U = max target length + 1) the recursions support: up to
// 32 warps of 256 label positions per utterance. Within it, a shape whose
// rings or registers do not fit one SM is reported as ASR_ERR_UNSUPPORTED
// before anything is launched (RNN-T: U up to about 3,200; TDT with durations
// 0..4: U up to about 4,000; durations 0..16: U up to about 1,000).
constexpr int kMaxLabelPositions = 8192;

// ---- asynchronous shared-memory prefetch of the next diagonal's lattice weights

__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"((uint32_t)__cvta_generic_to_shared(smem)),
                 "l"(gmem)
                 : "memory");
}

__device__ __forceinline__ void cp_async8(void* smem, const void* gmem) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"((uint32_t)__cvta_generic_to_shared(smem)),
                 "l"(gmem)
                 : "memory");
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

// Waits until at most one committed group (the newest prefetch) is still in flight.
__device__ __forceinline__ void cp_async_wait_prev() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

// Largest supported max_duration of the TDT recursions.
constexpr int kTdtMaxDuration = 16;
// Largest supported number of duration classes.
constexpr int kTdtMaxDurClasses = 32;

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

// The lattice weights (lpb, lpy, lpd) are read diagonal-major (diag_index) and
// alpha / beta are written diagonal-major, float64; log P(y|x) for the backward
// posteriors is recomputed from alpha rather than read from the fp32 output. The
// backward writes cb, ct (and gdur) node-major, for the backward joint.
int launch_rnnt_alpha(const LatticeMeta& m, int B, int U, const float* lpb, const float* lpy, double* alpha,
                      float* log_prob, float* loss, cudaStream_t st);
// `beta` is scratch of the TDT alpha array's size (sum over b of (T_b + 1) * U_b),
// read back only by label axes too long for the shared-memory rings.
int launch_rnnt_beta(const LatticeMeta& m, int B, int U, const float* lpb, const float* lpy, const double* alpha,
                     const float* grad_loss, float* cb, float* ct, double* beta, cudaStream_t st);

int launch_tdt_alpha(const LatticeMeta& m, int B, int U, int max_duration, const int32_t* durations, int n_dur,
                     int has_zero, const float* lpb, const float* lpy, const float* lpd, double* alpha,
                     float* log_prob, float* loss, cudaStream_t st);
// `beta` is scratch of the alpha array's size (sum over b of (T_b + 1) * U_b).
int launch_tdt_beta(const LatticeMeta& m, int B, int U, int max_duration, const int32_t* durations, int n_dur,
                    int has_zero, const float* lpb, const float* lpy, const float* lpd, const double* alpha,
                    const float* grad_loss, float* cb, float* ct, float* gdur, double* beta, cudaStream_t st);

}  // namespace asr
