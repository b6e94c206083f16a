// bf16 tcgen05 joint network (tf32 != 0, the systems' setting).
//
// Forward kernel (and the recompute pass of the backward), one persistent CTA
// per SM over 128-node tiles of the compact lattice:
//   warp 0      TMA producer: [joint_W; joint_W_dur] bf16 slices (32 K x 256 N,
//               64 B swizzle) into a 4-stage ring;
//   warp 1      MMA issuer (one thread): tcgen05.mma kind::f16, M = 128 nodes,
//               N = 256 vocabulary columns per chunk, fp32 accumulation in a
//               double-buffered TMEM accumulator (2 x 256 columns);
//   warps 2-9   A producers: hidden = tanh(enc + dec) for the tile, converted
//               to bf16 straight into the 128 B swizzled K-major smem layout the
//               MMA reads (all of K stays resident while the tile's vocabulary
//               chunks stream past; each K chunk is released to the next tile as
//               soon as the tile's last vocabulary chunk has consumed it);
//   warps 10-13 epilogue: one node per thread (TMEM lane = tile row). The
//               forward folds each chunk into an online log-sum-exp and gathers
//               the blank, label and duration logits: only the per-node lattice
//               weights reach HBM, never the logits. The backward variant turns
//               the recomputed logits into d loss / d logits (bf16 rows of G) and
//               the producers also store the bf16 hidden rows (H) for dW.
// Every mbarrier wait is bounded; a timeout sets the kernel's error word and the
// CTA drains its own TMA and MMA work, frees its TMEM and returns.
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "joint.cuh"
#include "tc_common.cuh"

namespace asr {
namespace {

using namespace tc;

constexpr int kBM = 128;                      // nodes per tile (UMMA M)
constexpr int kAK = 64;                       // K width of one A chunk (128 B rows)
constexpr int kBK = 32;                       // K width of one B stage (64 B rows)
constexpr int kNC = 256;                      // vocabulary columns per chunk (UMMA N)
constexpr int kMaxKChunks = 10;               // d rounded up to 64 must be <= 640
constexpr int kStages = 4;
constexpr int kProducerWarps = 8;
constexpr int kThreads = 32 * (2 + kProducerWarps + 4);  // TMA, MMA, producers, epilogue
constexpr int kAChunkBytes = kBM * kAK * 2;   // 16 KB
constexpr int kBStageBytes = kNC * kBK * 2;   // 16 KB
constexpr int kMaxDurCols = 16;
constexpr int kTmemCols = 512;

struct Geom {
    int kchunks;  // ceil(d / 64)
    int kpad;     // kchunks * 64
    int vpad;     // ceil((V + n_dur) / 16) * 16
    int nfull;    // full 256-column chunks
    int tail;     // width of the remaining chunk (multiple of 16), 0 if none
    int nchunks;  // nfull + (tail > 0)
};

Geom make_geom(const JointArgs& a) {
    Geom g;
    g.kchunks = (a.d + kAK - 1) / kAK;
    g.kpad = g.kchunks * kAK;
    g.vpad = (a.V + a.n_dur + 15) / 16 * 16;
    g.nfull = g.vpad / kNC;
    g.tail = g.vpad - g.nfull * kNC;
    g.nchunks = g.nfull + (g.tail > 0 ? 1 : 0);
    return g;
}

// Chunk j of a tile: the narrow tail chunk (if any) runs first, so that the
// last chunk of every tile is a full 256-wide one that overlaps the next tile's
// A production.
__device__ __forceinline__ void chunk_of(const Geom& g, int j, int& col, int& width) {
    if (g.tail > 0) {
        if (j == 0) {
            col = g.nfull * kNC;
            width = g.tail;
        } else {
            col = (j - 1) * kNC;
            width = kNC;
        }
    } else {
        col = j * kNC;
        width = kNC;
    }
}

struct Smem {
    uint8_t* a;         // kchunks x 16 KB
    uint8_t* b;         // kStages x 16 KB
    uint64_t* b_full;   // [kStages]
    uint64_t* b_empty;  // [kStages]
    uint64_t* a_full;   // [kMaxKChunks]
    uint64_t* a_empty;  // [kMaxKChunks]
    uint64_t* t_full;   // [2]
    uint64_t* t_empty;  // [2]
    uint64_t* done;     // [1]
    uint32_t* tmem_slot;
};

__host__ __device__ constexpr size_t smem_bytes_for(int kchunks) {
    return 1024 /* alignment slack */ + (size_t)kchunks * kAChunkBytes + (size_t)kStages * kBStageBytes +
           8 * (2 * kStages + 2 * kMaxKChunks + 5) + 16;
}

__device__ __forceinline__ Smem carve_smem(uint8_t* raw, int kchunks) {
    Smem s;
    uint8_t* p = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
    s.a = p;
    p += (size_t)kchunks * kAChunkBytes;
    s.b = p;
    p += (size_t)kStages * kBStageBytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(p);
    s.b_full = bars;
    s.b_empty = bars + kStages;
    s.a_full = bars + 2 * kStages;
    s.a_empty = bars + 2 * kStages + kMaxKChunks;
    s.t_full = bars + 2 * kStages + 2 * kMaxKChunks;
    s.t_empty = s.t_full + 2;
    s.done = s.t_empty + 2;
    s.tmem_slot = reinterpret_cast<uint32_t*>(s.done + 1);
    return s;
}

// Per-pass node range of the backward (pass p covers [bounds[2p], bounds[2p+1])).
struct PassRange {
    const int32_t* bounds;
    int pass;
};

struct TcParams {
    JointArgs a;
    Geom g;
    JointFwdOut fwd;  // forward outputs
    JointBwdIn bwd;   // backward inputs
    __nv_bfloat16* G;  // backward: (pass nodes, vpad) d loss / d logits
    __nv_bfloat16* H;  // backward: (pass nodes, kpad) hidden
    PassRange range;   // backward pass
    int* err;
};

__device__ __forceinline__ void node_range(const TcParams& P, bool bwd, int& begin, int& end) {
    const int N = total_nodes(P.a.m, P.a.B);
    if (!bwd) {
        begin = 0;
        end = N;
    } else {
        begin = min(P.range.bounds[2 * P.range.pass], N);
        end = min(P.range.bounds[2 * P.range.pass + 1], N);
    }
}

template <bool kBwd>
__global__ void __launch_bounds__(kThreads, 1)
    tc_joint_kernel(const __grid_constant__ CUtensorMap map_full, const __grid_constant__ CUtensorMap map_tail,
                    TcParams P) {
    extern __shared__ uint8_t smem_raw[];
    const Geom g = P.g;
    Smem sm = carve_smem(smem_raw, g.kchunks);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int* err = P.err;

    int begin, end;
    node_range(P, kBwd, begin, end);
    const int ntiles = end > begin ? (end - begin + kBM - 1) / kBM : 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&sm.b_full[s], 1);
            mbar_init(&sm.b_empty[s], 1);
        }
        for (int k = 0; k < kMaxKChunks; ++k) {
            mbar_init(&sm.a_full[k], kProducerWarps);
            mbar_init(&sm.a_empty[k], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&sm.t_full[i], 1);
            mbar_init(&sm.t_empty[i], 4);
        }
        mbar_init(sm.done, 1);
        fence_barrier_init();
        prefetch_tensormap(&map_full);
        prefetch_tensormap(&map_tail);
    }
    if (warp == 1) tmem_alloc(sm.tmem_slot, kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *sm.tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued_parity[kStages];
            bool issued[kStages];
#pragma unroll
            for (int s = 0; s < kStages; ++s) issued[s] = false, issued_parity[s] = 0;
            bool ok = true;
            for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
                for (int j = 0; ok && j < g.nchunks; ++j) {
                    int col, width;
                    chunk_of(g, j, col, width);
                    for (int ks = 0; ks < 2 * g.kchunks; ++ks) {
                        if (!mbar_wait(&sm.b_empty[stage], phase ^ 1, err, 1)) {
                            ok = false;
                            break;
                        }
                        mbar_arrive_expect_tx(&sm.b_full[stage], (uint32_t)width * kBK * 2);
                        tma_load_2d(sm.b + (size_t)stage * kBStageBytes, width == kNC ? &map_full : &map_tail,
                                    ks * kBK, col, &sm.b_full[stage]);
                        issued[stage] = true;
                        issued_parity[stage] = phase;
                        if (++stage == kStages) {
                            stage = 0;
                            phase ^= 1;
                        }
                    }
                }
            }
            // drain: every issued copy has landed before the CTA may exit
#pragma unroll
            for (int s = 0; s < kStages; ++s)
                if (issued[s]) mbar_wait(&sm.b_full[s], issued_parity[s], err, 2);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            const uint32_t idesc_full = idesc_bf16(kBM, kNC, false, false);
            const uint32_t idesc_tail = idesc_bf16(kBM, g.tail > 0 ? g.tail : 16, false, false);
            const uint32_t a_base = smem_u32(sm.a), b_base = smem_u32(sm.b);
            int stage = 0;
            uint32_t phase = 0;
            uint32_t q = 0;
            uint32_t it = 0;
            bool ok = true;
            for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x, ++it) {
                for (int j = 0; ok && j < g.nchunks; ++j, ++q) {
                    int col, width;
                    chunk_of(g, j, col, width);
                    const uint32_t buf = q & 1;
                    if (!mbar_wait(&sm.t_empty[buf], ((q >> 1) & 1) ^ 1, err, 3)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d_tmem = tmem_base + buf * kNC;
                    const uint32_t idesc = width == kNC ? idesc_full : idesc_tail;
                    for (int ks = 0; ks < 2 * g.kchunks; ++ks) {
                        const int kc = ks >> 1;
                        if (j == 0 && (ks & 1) == 0 && !mbar_wait(&sm.a_full[kc], it & 1, err, 4)) {
                            ok = false;
                            break;
                        }
                        if (!mbar_wait(&sm.b_full[stage], phase, err, 5)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
#pragma unroll
                        for (int kk = 0; kk < 2; ++kk) {
                            const uint64_t ad =
                                desc_k128(a_base + kc * kAChunkBytes + (uint32_t)(((ks & 1) * 2 + kk) * 32));
                            const uint64_t bd = desc_k64(b_base + stage * kBStageBytes + kk * 32);
                            mma_bf16(d_tmem, ad, bd, idesc, (ks | kk) != 0 ? 1u : 0u);
                        }
                        mma_commit(&sm.b_empty[stage]);
                        if (j == g.nchunks - 1 && (ks & 1)) mma_commit(&sm.a_empty[kc]);
                        if (++stage == kStages) {
                            stage = 0;
                            phase ^= 1;
                        }
                    }
                    if (ok) mma_commit(&sm.t_full[buf]);
                }
            }
            // drain: all issued MMAs complete before TMEM is released
            mma_commit(sm.done);
            mbar_wait(sm.done, 0, err, 6);
        }
    } else if (warp < 2 + kProducerWarps) {
        // ---------------------------------------------------------- A producers
        // Two threads per tile row, each building 32 of the 64 K columns of every
        // chunk: all 16 float4 loads of a half-chunk are issued before any tanh so
        // each thread keeps 256 bytes in flight.
        const int p = threadIdx.x - 64;  // 0..255
        const int r = p & (kBM - 1);     // tile row
        const int half = p >> 7;         // which 32 columns of each 64-wide chunk
        const int row_off = (r >> 3) * 1024 + (r & 7) * 128;
        const bool vec4 = (P.a.d & 3) == 0;
        uint32_t it = 0;
        bool ok = true;
        for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x, ++it) {
            const int n = begin + tile * kBM + r;
            const bool valid = n < end;
            int64_t eo = 0, dofs = 0;
            if (valid) {
                const NodeCoord c = node_coord(P.a.m, P.a.B, n);
                eo = ((int64_t)c.b * P.a.T + c.t) * P.a.d;
                dofs = ((int64_t)c.b * P.a.U + c.u) * P.a.d;
            }
            const float* er = P.a.enc + eo;
            const float* dr = P.a.dec + dofs;
            for (int kc = 0; kc < g.kchunks; ++kc) {
                if (it > 0 && !mbar_wait(&sm.a_empty[kc], (it - 1) & 1, err, 7)) {
                    ok = false;
                    break;
                }
                uint8_t* arow = sm.a + (size_t)kc * kAChunkBytes + row_off;
                const int kbase = kc * kAK + half * 32;
                float h[32];
                if (valid && vec4 && kbase + 32 <= P.a.d) {
                    float4 e[8], dd[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        e[i] = __ldg(reinterpret_cast<const float4*>(er + kbase) + i);
                        dd[i] = __ldg(reinterpret_cast<const float4*>(dr + kbase) + i);
                    }
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        h[4 * i + 0] = tanh_fast(e[i].x + dd[i].x);
                        h[4 * i + 1] = tanh_fast(e[i].y + dd[i].y);
                        h[4 * i + 2] = tanh_fast(e[i].z + dd[i].z);
                        h[4 * i + 3] = tanh_fast(e[i].w + dd[i].w);
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        const int k = kbase + i;
                        h[i] = (valid && k < P.a.d) ? tanh_fast(__ldg(er + k) + __ldg(dr + k)) : 0.f;
                    }
                }
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int u = half * 4 + q;  // 16-byte unit within the 128-byte row
                    uint4 w;
                    w.x = pack_bf16(h[8 * q + 0], h[8 * q + 1]);
                    w.y = pack_bf16(h[8 * q + 2], h[8 * q + 3]);
                    w.z = pack_bf16(h[8 * q + 4], h[8 * q + 5]);
                    w.w = pack_bf16(h[8 * q + 6], h[8 * q + 7]);
                    *reinterpret_cast<uint4*>(arow + ((u ^ (r & 7)) << 4)) = w;
                    if (kBwd && valid) *reinterpret_cast<uint4*>(P.H + (int64_t)(n - begin) * g.kpad + kbase + 8 * q) = w;
                }
                fence_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&sm.a_full[kc]);
            }
        }
    } else {
        // --------------------------------------------------------------- epilogue
        const int lane_base = 32 * (warp & 3);
        const int row = lane_base + lane;
        const JointArgs& a = P.a;
        const int Vf = a.V + a.n_dur;
        uint32_t q = 0;
        bool ok = true;
        for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
            const int n = begin + tile * kBM + row;
            const bool valid = n < end;
            int y = -1;
            if (valid) {
                const NodeCoord c = node_coord(a.m, a.B, n);
                y = (c.u < c.Ub - 1) ? __ldg(a.targets + (int64_t)c.b * a.S + c.u) : -1;
            }
            // forward state
            float m = -INFINITY, s = 0.f, lb = 0.f, ly = 0.f;
            float dur[kMaxDurCols];
#pragma unroll
            for (int k = 0; k < kMaxDurCols; ++k) dur[k] = 0.f;
            // backward per-node coefficients
            float lse = 0.f, cb = 0.f, ct = 0.f;
            if (kBwd && valid) {
                lse = P.bwd.lse[n];
                cb = P.bwd.cb[n];
                ct = P.bwd.ct[n];
            }
            for (int j = 0; j < g.nchunks; ++j, ++q) {
                int col, width;
                chunk_of(g, j, col, width);
                const uint32_t buf = q & 1;
                if (!mbar_wait(&sm.t_full[buf], (q >> 1) & 1, err, 8)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t taddr = tmem_base + ((uint32_t)lane_base << 16) + buf * kNC;
                for (int gi = 0; gi < width / 16; ++gi) {
                    float v[16];
                    tmem_ld16(taddr + gi * 16, v);
                    const int c0 = col + gi * 16;
                    if (!kBwd) {
                        if (c0 + 16 <= a.V) {
                            float gm = v[0];
#pragma unroll
                            for (int i = 1; i < 16; ++i) gm = fmaxf(gm, v[i]);
                            if (gm > m) {
                                s = (m == -INFINITY) ? 0.f : s * __expf(m - gm);
                                m = gm;
                            }
#pragma unroll
                            for (int i = 0; i < 16; ++i) s += __expf(v[i] - m);
#pragma unroll
                            for (int i = 0; i < 16; ++i) {
                                if (c0 + i == a.blank) lb = v[i];
                                if (c0 + i == y) ly = v[i];
                            }
                        } else {
#pragma unroll
                            for (int i = 0; i < 16; ++i) {
                                const int c = c0 + i;
                                if (c < a.V) {
                                    if (v[i] > m) {
                                        s = (m == -INFINITY) ? 0.f : s * __expf(m - v[i]);
                                        m = v[i];
                                    }
                                    s += __expf(v[i] - m);
                                    if (c == a.blank) lb = v[i];
                                    if (c == y) ly = v[i];
                                } else if (c < Vf) {
#pragma unroll
                                    for (int k = 0; k < kMaxDurCols; ++k)
                                        if (c - a.V == k) dur[k] = v[i];
                                }
                            }
                        }
                    } else if (valid) {
                        const float Pn = cb + ct;
                        float gv[16];
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            const int c = c0 + i;
                            float x = 0.f;
                            if (c < a.V) {
                                x = __expf(v[i] - lse) * Pn;
                                if (c == a.blank) x -= cb;
                                if (c == y) x -= ct;
                            } else if (c < Vf) {
                                x = P.bwd.gdur[(int64_t)n * a.n_dur + (c - a.V)];
                            }
                            gv[i] = x;
                        }
                        uint4 w0, w1;
                        w0.x = pack_bf16(gv[0], gv[1]);
                        w0.y = pack_bf16(gv[2], gv[3]);
                        w0.z = pack_bf16(gv[4], gv[5]);
                        w0.w = pack_bf16(gv[6], gv[7]);
                        w1.x = pack_bf16(gv[8], gv[9]);
                        w1.y = pack_bf16(gv[10], gv[11]);
                        w1.z = pack_bf16(gv[12], gv[13]);
                        w1.w = pack_bf16(gv[14], gv[15]);
                        uint4* dst = reinterpret_cast<uint4*>(P.G + (int64_t)(n - begin) * g.vpad + c0);
                        dst[0] = w0;
                        dst[1] = w1;
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&sm.t_empty[buf]);
            }
            if (!kBwd && ok && valid) {
                const float l = m + __logf(s);
                P.fwd.lse[n] = l;
                P.fwd.lpb[n] = lb - l - a.sigma;
                P.fwd.lpy[n] = y >= 0 ? ly - l - a.sigma : kNeg;
                if (a.n_dur > 0) {
                    float md = -INFINITY;
#pragma unroll
                    for (int k = 0; k < kMaxDurCols; ++k)
                        if (k < a.n_dur) md = fmaxf(md, dur[k]);
                    float sd = 0.f;
#pragma unroll
                    for (int k = 0; k < kMaxDurCols; ++k)
                        if (k < a.n_dur) sd += __expf(dur[k] - md);
                    const float lz = md + __logf(sd);
#pragma unroll
                    for (int k = 0; k < kMaxDurCols; ++k)
                        if (k < a.n_dur) P.fwd.lpd[(int64_t)n * a.n_dur + k] = dur[k] - lz;
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem_base, kTmemCols);
}

// [joint_W; joint_W_dur] -> bf16 (vpad, kpad), zero padded; optionally also the
// transpose (kpad, vpad) used as the K-major B operand of dH.
__global__ void prep_weights_kernel(const float* __restrict__ W, const float* __restrict__ Wd, int V, int n_dur,
                                    int d, int vpad, int kpad, __nv_bfloat16* __restrict__ Wf,
                                    __nv_bfloat16* __restrict__ Wt) {
    const int64_t total = (int64_t)vpad * kpad;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int r = (int)(i / kpad), k = (int)(i % kpad);
        float x = 0.f;
        if (k < d) {
            if (r < V)
                x = W[(int64_t)r * d + k];
            else if (r < V + n_dur)
                x = Wd[(int64_t)(r - V) * d + k];
        }
        const __nv_bfloat16 b = __float2bfloat16_rn(x);
        Wf[i] = b;
        if (Wt) Wt[(int64_t)k * vpad + r] = b;
    }
}

// ------------------------------------------------------------ host utilities

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// 2-D bf16 tensor map over a row-major (rows, cols) matrix, box (box_cols x box_rows).
bool make_map(CUtensorMap* map, const void* base, int rows, int cols, int box_cols, int box_rows,
              CUtensorMapSwizzle swz) {
    auto enc = tensor_map_encoder();
    if (!enc) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

size_t al256(size_t x) { return (x + 255) & ~size_t(255); }

int dyn_smem_limit() {
    int dev = 0, v = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    return v;
}

}  // namespace

bool tc_supported(const JointArgs& a) {
    const Geom g = make_geom(a);
    return g.kchunks <= kMaxKChunks && a.n_dur <= kMaxDurCols && tensor_map_encoder() != nullptr &&
           (int)smem_bytes_for(g.kchunks) <= dyn_smem_limit();
}

// Forward scratch: bf16 weights + the kernel error word.
size_t tc_forward_scratch_bytes(const JointArgs& a) {
    const Geom g = make_geom(a);
    return al256(sizeof(__nv_bfloat16) * (size_t)g.vpad * g.kpad) + 256;
}

int tc_joint_forward(const JointArgs& a, const JointFwdOut& o, void* scratch, size_t scratch_bytes,
                     cudaStream_t st) {
    const Geom g = make_geom(a);
    if (scratch_bytes < tc_forward_scratch_bytes(a)) return ASR_ERR_WORKSPACE;
    auto* Wf = reinterpret_cast<__nv_bfloat16*>(scratch);
    int* err = reinterpret_cast<int*>(reinterpret_cast<char*>(scratch) + al256(sizeof(__nv_bfloat16) * (size_t)g.vpad * g.kpad));
    ASR_CUDA_TRY(cudaMemsetAsync(err, 0, sizeof(int), st));
    {
        KernelTimer kt("joint_prep_weights", st);
        prep_weights_kernel<<<sm_count() * 4, 256, 0, st>>>(a.W, a.Wd, a.V, a.n_dur, a.d, g.vpad, g.kpad, Wf,
                                                             nullptr);
        ASR_LAUNCH_CHECK();
    }
    CUtensorMap mfull, mtail;
    if (!make_map(&mtail, Wf, g.vpad, g.kpad, kBK, g.tail > 0 ? g.tail : 16, CU_TENSOR_MAP_SWIZZLE_64B))
        return ASR_ERR_CUDA;
    if (g.nfull == 0)
        mfull = mtail;
    else if (!make_map(&mfull, Wf, g.vpad, g.kpad, kBK, kNC, CU_TENSOR_MAP_SWIZZLE_64B))
        return ASR_ERR_CUDA;
    TcParams P;
    std::memset(&P, 0, sizeof(P));
    P.a = a;
    P.g = g;
    P.fwd = o;
    P.err = err;
    const size_t smem = smem_bytes_for(g.kchunks);
    ASR_CUDA_TRY(cudaFuncSetAttribute(tc_joint_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    const int64_t cap_tiles = ((int64_t)a.B * a.T * a.U + kBM - 1) / kBM;
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(cap_tiles, sm_count()));
    KernelTimer kt("joint_fwd_tc", st);
    tc_joint_kernel<false><<<grid, kThreads, smem, st>>>(mfull, mtail, P);
    ASR_LAUNCH_CHECK();
    return ASR_OK;
}

bool tc_backward_supported(const JointArgs&) { return false; }
size_t tc_backward_scratch_bytes(const JointArgs&, int) { return 0; }
int tc_joint_backward(const JointArgs&, const JointBwdIn&, const JointBwdOut&, int, void*, size_t, cudaStream_t) {
    return ASR_ERR_UNSUPPORTED;
}

}  // namespace asr
