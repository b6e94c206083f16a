// Shared device helpers for the sequence-loss kernels (sm_100a).
//
// Lattice storage convention used by every transducer kernel in this library:
// only valid nodes are stored ("compact" layout). Utterance b owns
//   T_b = in_lens[b] frames and U_b = tgt_lens[b] + 1 label positions,
// node (b, t, u) with t < T_b, u < U_b lives at  off[b] + t * U_b + u,
// and the TDT forward variable, defined on the (T_b + 1)-frame grid, lives at
//   aoff[b] + t * U_b + u  for t <= T_b.
// off / aoff are exclusive prefix sums computed on the device (no host sync),
// so padded lattice nodes cost neither compute nor memory traffic.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "asr_b200.h"
#include "profiler.cuh"

namespace asr {

// Finite "log zero" of the reference transducer kernels (rnnt.cu:35, tdt.cu:43):
// exp(NEG - x) underflows to 0 and NEG + NEG stays finite.
constexpr float kNeg = -1e30f;

__device__ __forceinline__ float lae(float a, float b) {
    // log(exp(a) + exp(b)); -inf safe, as ctc.cu:38-43.
    const float m = fmaxf(a, b);
    if (m == -INFINITY) return -INFINITY;
    return m + log1pf(__expf(-fabsf(a - b)));
}

// Mixed-precision log-add for the lattice recursions. The running forward /
// backward variables reach |alpha| ~ 10^3 on long lattices, where one fp32 ulp
// is ~1e-4 and rounding accumulates along T + U steps. The recursion state is
// therefore kept in float64; only the bounded correction term
// log1p(exp(-|a - b|)) in [0, log 2] is evaluated in fp32.
__device__ __forceinline__ double lae_d(double a, double b) {
    const double m = fmax(a, b);
    if (m == -INFINITY) return -INFINITY;
    const float d = (float)(fmin(a, b) - m);
    return m + (double)__logf(1.f + __expf(d));
}

// Running log-sum-exp of float64 terms: max first, then one exp per term and a
// single log (the terms of one lattice node are all known before the sum).
// The max and the sum are pairwise trees, so the dependent chain of a node is
// log2(N) deep rather than N.
template <int N>
__device__ __forceinline__ double lse_d(const double (&x)[N]) {
    double mx[N];
#pragma unroll
    for (int i = 0; i < N; ++i) mx[i] = x[i];
#pragma unroll
    for (int w = 1; w < N; w *= 2)
#pragma unroll
        for (int i = 0; i + w < N; i += 2 * w) mx[i] = fmax(mx[i], mx[i + w]);
    const double m = mx[0];
    if (m <= -1e29) return m;  // every term is the finite log-zero sentinel
    float e[N];
#pragma unroll
    for (int i = 0; i < N; ++i) e[i] = __expf((float)(x[i] - m));
#pragma unroll
    for (int w = 1; w < N; w *= 2)
#pragma unroll
        for (int i = 0; i + w < N; i += 2 * w) e[i] += e[i + w];
    return m + (double)__logf(e[0]);
}

// Diagonal-major order of a rows x cols lattice grid: anti-diagonals g = t + u
// in order, u ascending within a diagonal. The recursions sweep anti-diagonals,
// so storing the per-node lattice weights and the forward / backward variables
// this way makes every diagonal one contiguous block (coalesced loads). Index
// of node (t, u) within the grid:
__host__ __device__ __forceinline__ int diag_index(int t, int u, int rows, int cols) {
    const int g = t + u;
    const int mn = rows < cols ? rows : cols, mx = rows < cols ? cols : rows;
    int s;
    if (g <= mn) {
        s = g * (g + 1) / 2;
    } else if (g <= mx) {
        s = mn * (mn + 1) / 2 + (g - mn) * mn;
    } else {
        const int h = rows + cols - 1 - g;
        s = rows * cols - h * (h + 1) / 2;
    }
    const int ulo = g - rows + 1 > 0 ? g - rows + 1 : 0;
    return s + u - ulo;
}

// Per-batch lattice bookkeeping produced by lattice_prep_kernel.
struct LatticeMeta {
    int32_t* Tb;    // (B,) clamped frames
    int32_t* Ub;    // (B,) clamped label positions (tgt_len + 1)
    int32_t* off;   // (B+1,) node offsets (T_b * U_b prefix)
    int32_t* aoff;  // (B+1,) TDT alpha offsets ((T_b + 1) * U_b prefix)
    int32_t* status;  // [0]: 1 when a length had to be clamped
};

// Bytes needed by LatticeMeta for a batch of B (256-byte aligned pieces).
inline size_t lattice_meta_bytes(int B) {
    auto al = [](size_t x) { return (x + 255) & ~size_t(255); };
    return al(sizeof(int32_t) * B) * 2 + al(sizeof(int32_t) * (B + 1)) * 2 + al(sizeof(int32_t) * 4);
}

// Carves a LatticeMeta out of `ws`; returns the first byte after it.
inline char* lattice_meta_carve(char* ws, int B, LatticeMeta* m) {
    auto al = [](size_t x) { return (x + 255) & ~size_t(255); };
    m->Tb = reinterpret_cast<int32_t*>(ws);
    ws += al(sizeof(int32_t) * B);
    m->Ub = reinterpret_cast<int32_t*>(ws);
    ws += al(sizeof(int32_t) * B);
    m->off = reinterpret_cast<int32_t*>(ws);
    ws += al(sizeof(int32_t) * (B + 1));
    m->aoff = reinterpret_cast<int32_t*>(ws);
    ws += al(sizeof(int32_t) * (B + 1));
    m->status = reinterpret_cast<int32_t*>(ws);
    ws += al(sizeof(int32_t) * 4);
    return ws;
}

// Utterance owning compact node n: largest b with off[b] <= n (off[0] = 0).
__device__ __forceinline__ int find_utt(const int32_t* __restrict__ off, int B, int n) {
    int lo = 0, hi = B - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (__ldg(off + mid) <= n)
            lo = mid;
        else
            hi = mid - 1;
    }
    return lo;
}

struct NodeCoord {
    int b, t, u, Ub;
};

__device__ __forceinline__ NodeCoord node_coord(const LatticeMeta& m, int B, int n) {
    NodeCoord c;
    c.b = find_utt(m.off, B, n);
    c.Ub = __ldg(m.Ub + c.b);
    const int r = n - __ldg(m.off + c.b);
    c.t = r / c.Ub;
    c.u = r - c.t * c.Ub;
    return c;
}

__device__ __forceinline__ int total_nodes(const LatticeMeta& m, int B) { return *((volatile int32_t*)m.off + B); }

// ---------------------------------------------------------------- launch helpers

#define ASR_CUDA_TRY(expr)                              \
    do {                                                \
        cudaError_t e_ = (expr);                        \
        if (e_ != cudaSuccess) return ASR_ERR_CUDA;     \
    } while (0)

#define ASR_LAUNCH_CHECK()                                  \
    do {                                                    \
        cudaError_t e_ = cudaGetLastError();                \
        if (e_ != cudaSuccess) return ASR_ERR_CUDA;         \
    } while (0)

inline int sm_count() {
    int dev = 0, n = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n;
}

// Host-side launchers defined in lattice.cu.
int launch_lattice_prep(const int32_t* in_lens, const int32_t* tgt_lens, int B, int T, int U, int S,
                        const LatticeMeta& m, cudaStream_t stream);
// CTC beta + gradient (ctc.cu). post_only = 1 writes grad_loss * (state posterior
// mass per column) instead of d loss / d logits.
int ctc_grad_dispatch(const double* alpha, const float* log_probs, const int32_t* targets, const int32_t* in_lens,
                      const int32_t* tgt_lens, const float* grad_loss, int zero_infinity, int post_only, int B, int T,
                      int V, int S, float* grad, cudaStream_t st);
// bf16 <-> fp32 element conversions of n contiguous values (bf16 activations and
// their gradients).
int launch_bf16_to_f32(const __nv_bfloat16* src, float* dst, int64_t n, cudaStream_t stream);
int launch_f32_to_bf16(const float* src, __nv_bfloat16* dst, int64_t n, cudaStream_t stream);

}  // namespace asr
