// Lattice bookkeeping: clamps the per-utterance lengths and builds the compact
// node offsets (exclusive prefix sums) on the device, one block per batch.
#include "common.cuh"

namespace asr {

namespace {

constexpr int kPrepThreads = 1024;

__global__ void __launch_bounds__(kPrepThreads)
    lattice_prep_kernel(const int32_t* __restrict__ in_lens, const int32_t* __restrict__ tgt_lens, int B, int T,
                        int U, int S, LatticeMeta m) {
    __shared__ int32_t warp_n[32], warp_a[32];
    __shared__ int32_t carry_n, carry_a, clamped;
    const int tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    if (tid == 0) {
        carry_n = 0;
        carry_a = 0;
        clamped = 0;
    }
    __syncthreads();
    const int umax = min(U - 1, S);  // a label position needs a target column
    for (int base = 0; base < B; base += kPrepThreads) {
        const int b = base + tid;
        int n = 0, a = 0;
        if (b < B) {
            const int ti = in_lens[b], gi = tgt_lens[b];
            const int tb = min(max(ti, 1), T);
            const int ub = min(max(gi, 0), max(umax, 0)) + 1;
            if (tb != ti || ub != gi + 1) atomicOr(&clamped, 1);
            m.Tb[b] = tb;
            m.Ub[b] = ub;
            n = tb * ub;
            a = (tb + 1) * ub;
        }
        // block-wide inclusive scan of (n, a)
        int sn = n, sa = a;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int yn = __shfl_up_sync(0xffffffffu, sn, o);
            const int ya = __shfl_up_sync(0xffffffffu, sa, o);
            if (lane >= o) {
                sn += yn;
                sa += ya;
            }
        }
        if (lane == 31) {
            warp_n[warp] = sn;
            warp_a[warp] = sa;
        }
        __syncthreads();
        if (warp == 0) {
            int wn = warp_n[lane], wa = warp_a[lane];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int yn = __shfl_up_sync(0xffffffffu, wn, o);
                const int ya = __shfl_up_sync(0xffffffffu, wa, o);
                if (lane >= o) {
                    wn += yn;
                    wa += ya;
                }
            }
            warp_n[lane] = wn;
            warp_a[lane] = wa;
        }
        __syncthreads();
        const int pre_n = (warp > 0 ? warp_n[warp - 1] : 0) + sn - n;
        const int pre_a = (warp > 0 ? warp_a[warp - 1] : 0) + sa - a;
        if (b < B) {
            m.off[b] = carry_n + pre_n;
            m.aoff[b] = carry_a + pre_a;
        }
        __syncthreads();
        if (tid == kPrepThreads - 1) {
            carry_n += pre_n + n;
            carry_a += pre_a + a;
        }
        __syncthreads();
    }
    if (tid == 0) {
        m.off[B] = carry_n;
        m.aoff[B] = carry_a;
        m.status[0] = clamped;
    }
}

// Grid-stride element conversions (bandwidth bound; 8 elements per thread step).
__global__ void bf16_to_f32_kernel(const __nv_bfloat16* __restrict__ src, float* __restrict__ dst, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = __bfloat162float(src[i]);
}

__global__ void f32_to_bf16_kernel(const float* __restrict__ src, __nv_bfloat16* __restrict__ dst, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = __float2bfloat16_rn(src[i]);
}

}  // namespace

int launch_bf16_to_f32(const __nv_bfloat16* src, float* dst, int64_t n, cudaStream_t stream) {
    if (n <= 0) return ASR_OK;
    KernelTimer kt("act_convert", stream);
    bf16_to_f32_kernel<<<sm_count() * 8, 256, 0, stream>>>(src, dst, n);
    ASR_LAUNCH_CHECK();
    return ASR_OK;
}

int launch_f32_to_bf16(const float* src, __nv_bfloat16* dst, int64_t n, cudaStream_t stream) {
    if (n <= 0) return ASR_OK;
    KernelTimer kt("act_convert", stream);
    f32_to_bf16_kernel<<<sm_count() * 8, 256, 0, stream>>>(src, dst, n);
    ASR_LAUNCH_CHECK();
    return ASR_OK;
}

int launch_lattice_prep(const int32_t* in_lens, const int32_t* tgt_lens, int B, int T, int U, int S,
                        const LatticeMeta& m, cudaStream_t stream) {
    KernelTimer kt("lattice_prep", stream);
    lattice_prep_kernel<<<1, kPrepThreads, 0, stream>>>(in_lens, tgt_lens, B, T, U, S, m);
    ASR_LAUNCH_CHECK();
    return ASR_OK;
}

}  // namespace asr
