// Launchers of the lattice recursions (dp_rnnt.cu, dp_tdt.cu).
#pragma once

#include "common.cuh"

namespace asr {

// Largest label axis (U = max target length + 1) the recursions support: one
// thread per label position in a CTA.
constexpr int kMaxLabelPositions = 1024;

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

// The forward variable is stored in float64 (see lae_d); log P(y|x) for the
// backward posteriors is recomputed from it rather than read from the fp32 output.
int launch_rnnt_alpha(const LatticeMeta& m, int B, int U, const float* lpb, const float* lpy, double* alpha,
                      float* log_prob, float* loss, cudaStream_t st);
int launch_rnnt_beta(const LatticeMeta& m, int B, int U, const float* lpb, const float* lpy, const double* alpha,
                     const float* grad_loss, float* cb, float* ct, cudaStream_t st);

int launch_tdt_alpha(const LatticeMeta& m, int B, int U, int max_duration, const int32_t* durations, int n_dur,
                     int has_zero, const float* lpb, const float* lpy, const float* lpd, double* alpha,
                     float* log_prob, float* loss, cudaStream_t st);
// `beta` is scratch of the alpha array's size (sum over b of (T_b + 1) * U_b).
int launch_tdt_beta(const LatticeMeta& m, int B, int U, int max_duration, const int32_t* durations, int n_dur,
                    int has_zero, const float* lpb, const float* lpy, const float* lpd, const double* alpha,
                    const float* grad_loss, float* cb, float* ct, float* gdur, double* beta, cudaStream_t st);

}  // namespace asr
