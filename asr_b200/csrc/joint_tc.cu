// bf16 tcgen05 joint network (tf32 != 0, the systems' setting).
//
// Forward kernel (and the recompute pass of the backward), one persistent CTA
// per SM over 128-node tiles of the compact lattice:
//   warp 0      TMA producer: [joint_W; joint_W_dur] bf16 slices (64 K x one
//               vocabulary chunk, 128 B swizzle: one large box per stage, the
//               box count rather than the bytes bounds TMA throughput) into a
//               2-stage ring;
//   warp 1      MMA issuer (one thread): tcgen05.mma kind::f16, M = 128 nodes,
//               N = one vocabulary chunk (<= 256 columns, e.g. 5 x 208 for
//               1029 columns), fp32 accumulation in a double-buffered TMEM
//               accumulator (2 x 256 columns). Optionally a CTA pair runs one
//               M = 256 MMA (cta_group::2), each CTA streaming half the weights;
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
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "joint.cuh"
#include "tc_common.cuh"

namespace asr {
namespace {

using namespace tc;

constexpr int kBM = 128;                      // nodes per tile (UMMA M)
constexpr int kAK = 64;                       // K width of one A chunk (128 B rows)
constexpr int kBK = 64;                       // K width of one B stage (128 B rows, = one A chunk)
constexpr int kNC = 256;                      // vocabulary columns per chunk (UMMA N)
constexpr int kMaxKChunks = 10;               // d rounded up to 64 must be <= 640
constexpr int kStages = 2;
constexpr int kEpilogueWarp0 = 4;                    // warps 4-7: epilogue (one TMEM lane quarter each)
constexpr int kThreads = 32 * (kEpilogueWarp0 + 4);  // weight TMA, MMA, hidden TMA, idle, epilogue
constexpr int kAChunkBytes = kBM * kAK * 2;   // 16 KB
constexpr int kBStageBytes = kNC * kBK * 2;   // 32 KB
constexpr int kMaxDurCols = 16;
constexpr int kTmemCols = 512;
constexpr int kMaxRing = 8;           // barrier slots per ring
constexpr int kStreamStagesMax = 6;
constexpr int kSmemBudget = 227 * 1024;
constexpr int kBarBytes = 8 * (2 * kMaxRing + 2 * kMaxKChunks + 5) + 16;

struct Geom {
    int parts;    // operand parts along K: 1 (bf16) or 3 (split fp32: hi, lo, hi)
    int kp;       // hidden columns of one part: ceil(d / 64) * 64
    int kchunks;  // 64-column K chunks of the hidden rows over all parts
    int kpad;     // parts * kp: width of the hidden rows H and of the weight rows Wf
    int vpad;     // ceil((V + n_dur) / 16) * 16
    int gw;       // parts * vpad: width of the G rows and of the transposed weight
    int cw;       // vocabulary columns of a chunk (multiple of 16, <= 256)
    int lw;       // columns of the last chunk (multiple of 16, <= cw)
    int nchunks;  // chunks per tile
    int sstage;   // streamed variant: bytes of one ring stage (hidden chunk + weight chunk)
    int nstream;  // streamed variant: ring stages
};

// Split fp32 mode (JointArgs::split): the operands are stored as K-blocks of
// their bf16 parts, paired so that every GEMM is unchanged over a longer K:
//   H  rows [H_hi | H_lo | H_hi]  with  Wf rows [W_hi | W_hi | W_lo]   (logits)
//   G  rows [G_hi | G_hi | G_lo]  with  Wt rows [Wt_hi | Wt_lo | Wt_hi] (d hidden)
//   dW = sum over blocks p of G_p^T H_p                                   (dW)
// so each product is hi*hi + lo*hi + hi*lo.
//
// The vocabulary is cut into equal chunks (e.g. 1040 = 5 x 208): every chunk
// runs the same number of full-width MMAs per weight stage, instead of a narrow
// remainder chunk paying a full ring of weight stages for a few columns.
Geom make_geom(const JointArgs& a) {
    Geom g;
    const int kd = a.d + (a.head && a.bias ? 1 : 0);  // CTC head: bias as a ones column
    g.parts = a.split ? 3 : 1;
    g.kp = (kd + kAK - 1) / kAK * kAK;
    g.kchunks = g.parts * (g.kp / kAK);
    g.kpad = g.parts * g.kp;
    g.vpad = (a.V + a.n_dur + 15) / 16 * 16;
    g.gw = g.parts * g.vpad;
    g.nchunks = (g.vpad + kNC - 1) / kNC;
    g.cw = ((g.vpad + g.nchunks - 1) / g.nchunks + 15) / 16 * 16;
    g.nchunks = (g.vpad + g.cw - 1) / g.cw;
    g.lw = g.vpad - (g.nchunks - 1) * g.cw;
    g.sstage = kAChunkBytes + g.cw * kBK * 2;  // a multiple of 2 KB: stage bases stay 1024-aligned
    g.nstream = std::min(kStreamStagesMax, (kSmemBudget - 1024 - kBarBytes) / g.sstage);
    if (const char* e = std::getenv("ASR_B200_JOINT_RING")) {  // tuning knob: fewer streamed stages
        const int r = std::atoi(e);
        if (r >= 2 && r < g.nstream) g.nstream = r;
    }
    return g;
}

__device__ __forceinline__ void chunk_of(const Geom& g, int j, int& col, int& width) {
    col = j * g.cw;
    width = j == g.nchunks - 1 ? g.lw : g.cw;
}

struct Smem {
    uint8_t* a;         // kchunks x 16 KB
    uint8_t* b;         // 64 KB weight ring (kStages x 16 KB, or 2 kStages x 8 KB for a pair)
    uint64_t* b_full;   // [2 kStages]
    uint64_t* b_empty;  // [2 kStages]
    uint64_t* a_full;   // [kMaxKChunks]
    uint64_t* a_empty;  // [kMaxKChunks]
    uint64_t* t_full;   // [2]
    uint64_t* t_empty;  // [2]
    uint64_t* done;     // [1]
    uint32_t* tmem_slot;
};

// Streamed-A variant (the default; required when d > 64 * kMaxKChunks, where
// the 128-row hidden tile no longer fits in shared memory): every ring stage
// carries one hidden chunk (16 KB) and one weight chunk (cw x 128 B), so the
// tile's hidden rows are re-read from L2 once per vocabulary chunk, and the ring
// gets as many stages as shared memory holds (5 of 42.5 KB at cw = 208). On B200
// this measured faster than keeping the hidden tile resident behind a 2-stage
// weight ring (d = 640, B = 128: dlogits 6.2 vs 6.8 ms, forward 4.4 vs 4.5 ms).

__host__ __device__ constexpr size_t smem_bytes_for(int kchunks, bool stream = false, int sstage = 0,
                                                    int nstream = 0) {
    return 1024 /* alignment slack */ +
           (stream ? (size_t)nstream * sstage : (size_t)kchunks * kAChunkBytes + (size_t)kStages * kBStageBytes) +
           kBarBytes;
}

__device__ __forceinline__ Smem carve_smem(uint8_t* raw, int kchunks, bool stream = false, int ring_bytes = 0) {
    Smem s;
    uint8_t* p = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
    s.a = p;
    if (stream) {
        s.b = p;
        p += (size_t)ring_bytes;
    } else {
        p += (size_t)kchunks * kAChunkBytes;
        s.b = p;
        p += (size_t)kStages * kBStageBytes;
    }
    uint64_t* bars = reinterpret_cast<uint64_t*>(p);
    s.b_full = bars;
    s.b_empty = bars + kMaxRing;
    s.a_full = bars + 2 * kMaxRing;
    s.a_empty = bars + 2 * kMaxRing + kMaxKChunks;
    s.t_full = bars + 2 * kMaxRing + 2 * kMaxKChunks;
    s.t_empty = s.t_full + 2;
    s.done = s.t_empty + 2;
    s.tmem_slot = reinterpret_cast<uint32_t*>(s.done + 1);
    return s;
}

// Per-pass node range of the backward (pass p covers [bounds[p], bounds[p+1])).
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
    PassRange range;   // node pass
    LogitStash stash;  // forward: written for nodes below stash.nodes; backward: those nodes are skipped
    int* err;
};

// Nodes [begin, end) of this launch within the pass that starts at `base` (the
// row origin of the pass's H and G buffers). The backward leaves the stashed
// nodes below stash.nodes to the stash kernel; base and stash.nodes are
// multiples of 256, so its tiles start on whole tiles of the pass.
__device__ __forceinline__ void node_range(const TcParams& P, bool bwd, int& base, int& begin, int& end) {
    const int N = total_nodes(P.a.m, P.a.B);
    base = min(P.range.bounds[P.range.pass], N);
    end = min(P.range.bounds[P.range.pass + 1], N);
    begin = bwd ? min(end, max(base, P.stash.nodes)) : base;
}

// B ring geometry per CTA: a pair splits each 256-column chunk, so every CTA
// streams half the weight bytes and keeps twice as many stages in flight.
template <int kCta>
__host__ __device__ constexpr int b_stage_bytes() { return kNC / kCta * kBK * 2; }
template <int kCta>
__host__ __device__ constexpr int b_stages() { return kStages * kCta; }

template <bool kBwd, int kCta, bool kStream, bool kStash = false>
__global__ void __launch_bounds__(kThreads, 1)
    tc_joint_kernel(const __grid_constant__ CUtensorMap map_full, const __grid_constant__ CUtensorMap map_tail,
                    const __grid_constant__ CUtensorMap map_h, TcParams P) {
    static_assert(!kStream || kCta == 1, "the streamed-A variant runs single CTAs");
    static_assert(!kStash || (!kBwd && kCta == 1), "the forward of single CTAs writes the logit stash");
    extern __shared__ uint8_t smem_raw[];
    const Geom g = P.g;
    const int SB = kStream ? g.sstage : b_stage_bytes<kCta>();
    const int NS = kStream ? g.nstream : b_stages<kCta>();
    Smem sm = carve_smem(smem_raw, g.kchunks, kStream, g.sstage * g.nstream);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int* err = P.err;
    const uint32_t rank = kCta == 2 ? cluster_ctarank() : 0;
    const bool leader = rank == 0;
    // work units: one 128-node tile (kCta = 1) or a pair of consecutive tiles,
    // tile 2p + rank in CTA `rank` (kCta = 2)
    const int unit0 = blockIdx.x / kCta, units_stride = gridDim.x / kCta;

    int base, begin, end;
    node_range(P, kBwd, base, begin, end);
    const int row_off = begin - base;  // pass-relative H / G row of this launch's first node
    const int ntiles = end > begin ? (end - begin + kBM - 1) / kBM : 0;
    const int nunits = (ntiles + kCta - 1) / kCta;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&sm.b_full[s], 1);
            mbar_init(&sm.b_empty[s], 1);
        }
        for (int k = 0; k < kMaxKChunks; ++k) {
            mbar_init(&sm.a_full[k], 1);  // the hidden-tile loader's expect_tx arrival
            mbar_init(&sm.a_empty[k], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&sm.t_full[i], 1);
            mbar_init(&sm.t_empty[i], 4 * kCta);
        }
        mbar_init(sm.done, 1);
        fence_barrier_init();
        prefetch_tensormap(&map_full);
        prefetch_tensormap(&map_tail);
        prefetch_tensormap(&map_h);
    }
    if (kCta == 2) {
        cluster_sync();  // both CTAs' barriers exist before any cross-CTA arrival
        if (warp == 1) tmem_alloc_pair(sm.tmem_slot, kTmemCols);
    } else if (warp == 1) {
        tmem_alloc(sm.tmem_slot, kTmemCols);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *sm.tmem_slot;
    // shared::cluster addresses of the pair's barriers
    auto in_leader = [&](uint64_t* bar) { return kCta == 2 ? mapa_shared(smem_u32(bar), 0) : smem_u32(bar); };
    auto in_peer = [&](uint64_t* bar) { return mapa_shared(smem_u32(bar), 1); };

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued_parity[kMaxRing];
            bool issued[kMaxRing];
#pragma unroll
            for (int s = 0; s < NS; ++s) issued[s] = false, issued_parity[s] = 0;
            bool ok = true;
            for (int unit = unit0; ok && unit < nunits; unit += units_stride) {
                for (int j = 0; ok && j < g.nchunks; ++j) {
                    int col, width;
                    chunk_of(g, j, col, width);
                    const int rows = width / kCta;  // weight rows this CTA supplies
                    for (int ks = 0; ks < g.kchunks; ++ks) {
                        if (!mbar_wait_cluster(&sm.b_empty[stage], phase ^ 1, err, 1)) {
                            ok = false;
                            break;
                        }
                        uint8_t* dst = sm.b + (size_t)stage * SB;
                        const CUtensorMap* map = width == g.cw ? &map_full : &map_tail;
                        if (kStream) {  // hidden chunk (tile rows x 64) then weight chunk
                            mbar_arrive_expect_tx(&sm.b_full[stage], kAChunkBytes + (uint32_t)width * kBK * 2);
                            tma_load_2d(dst, &map_h, ks * kAK, row_off + unit * kBM, &sm.b_full[stage]);
                            tma_load_2d(dst + kAChunkBytes, map, ks * kBK, col, &sm.b_full[stage]);
                        } else if (kCta == 2) {
                            if (leader) mbar_arrive_expect_tx(&sm.b_full[stage], (uint32_t)width * kBK * 2);
                            tma_load_2d_pair(dst, map, ks * kBK, col + (int)rank * rows, in_leader(&sm.b_full[stage]));
                        } else {
                            mbar_arrive_expect_tx(&sm.b_full[stage], (uint32_t)width * kBK * 2);
                            tma_load_2d(dst, map, ks * kBK, col, &sm.b_full[stage]);
                        }
                        issued[stage] = true;
                        issued_parity[stage] = phase;
                        if (++stage == NS) {
                            stage = 0;
                            phase ^= 1;
                        }
                    }
                }
            }
            // drain: every issued copy has landed before the CTA may exit (for a
            // pair the even CTA's full barrier counts both halves)
            if (leader) {
#pragma unroll
                for (int s = 0; s < NS; ++s)
                    if (issued[s]) mbar_wait_cluster(&sm.b_full[s], issued_parity[s], err, 2);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------- MMA issuer
        if (lane == 0 && leader) {
            const uint32_t idesc_full = idesc_bf16(kBM * kCta, g.cw, false, false);
            const uint32_t idesc_tail = idesc_bf16(kBM * kCta, g.lw, false, false);
            const uint32_t a_base = smem_u32(sm.a), b_base = smem_u32(sm.b);
            auto commit_both = [&](uint64_t* bar) {
                if (kCta == 2) {
                    mma_commit_pair(smem_u32(bar));
                    mma_commit_pair(in_peer(bar));
                } else {
                    mma_commit(bar);
                }
            };
            int stage = 0;
            uint32_t phase = 0;
            uint32_t q = 0;
            uint32_t it = 0;
            bool ok = true;
            for (int unit = unit0; ok && unit < nunits; unit += units_stride, ++it) {
                for (int j = 0; ok && j < g.nchunks; ++j, ++q) {
                    int col, width;
                    chunk_of(g, j, col, width);
                    const uint32_t buf = q & 1;
                    if (!mbar_wait_cluster(&sm.t_empty[buf], ((q >> 1) & 1) ^ 1, err, 3)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d_tmem = tmem_base + buf * kNC;
                    const uint32_t idesc = width == g.cw ? idesc_full : idesc_tail;
                    for (int kc = 0; kc < g.kchunks; ++kc) {
                        if (!kStream && j == 0 && !mbar_wait_cluster(&sm.a_full[kc], it & 1, err, 4)) {
                            ok = false;
                            break;
                        }
                        if (!mbar_wait_cluster(&sm.b_full[stage], phase, err, 5)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
#pragma unroll
                        for (int kk = 0; kk < kBK / 16; ++kk) {
                            const uint32_t sa = kStream ? b_base + stage * SB : a_base + kc * kAChunkBytes;
                            const uint32_t sb = b_base + stage * SB + (kStream ? kAChunkBytes : 0);
                            const uint64_t ad = desc_k128(sa + kk * 32);
                            const uint64_t bd = desc_k128(sb + kk * 32);
                            if (kCta == 2)
                                mma_bf16_pair(d_tmem, ad, bd, idesc, (kc | kk) != 0 ? 1u : 0u);
                            else
                                mma_bf16(d_tmem, ad, bd, idesc, (kc | kk) != 0 ? 1u : 0u);
                        }
                        commit_both(&sm.b_empty[stage]);
                        if (!kStream && j == g.nchunks - 1) commit_both(&sm.a_empty[kc]);
                        if (++stage == NS) {
                            stage = 0;
                            phase ^= 1;
                        }
                    }
                    if (ok) commit_both(&sm.t_full[buf]);
                }
            }
            // drain: all issued MMAs complete before either CTA releases its TMEM
            commit_both(sm.done);
            mbar_wait(sm.done, 0, err, 6);
        } else if (lane == 0) {
            mbar_wait_cluster(sm.done, 0, err, 6);  // odd CTA: the even CTA's MMAs write this TMEM
        }
    } else if (warp == 2) {
        // ------------------------------------------------------- hidden-tile TMA
        // The tile's rows of H = bf16(tanh(enc + dec)) (written by hidden_kernel
        // for this pass) into the resident 128 B swizzled K chunks; chunk kc of
        // the next tile is reloaded as soon as the last vocabulary chunk of the
        // current tile has consumed it. (The streamed variant loads them with the
        // weights instead.)
        if (!kStream && lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            bool issued[kMaxKChunks];
            uint32_t ipar[kMaxKChunks];
#pragma unroll
            for (int k = 0; k < kMaxKChunks; ++k) issued[k] = false, ipar[k] = 0;
            for (int unit = unit0; ok && unit < nunits; unit += units_stride, ++it) {
                const int row0 = row_off + (unit * kCta + (int)rank) * kBM;  // pass-relative H row
                for (int kc = 0; kc < g.kchunks; ++kc) {
                    if (it > 0 && !mbar_wait_cluster(&sm.a_empty[kc], (it - 1) & 1, err, 7)) {
                        ok = false;
                        break;
                    }
                    uint8_t* dst = sm.a + (size_t)kc * kAChunkBytes;
                    if (kCta == 2) {
                        if (leader) mbar_arrive_expect_tx(&sm.a_full[kc], 2 * kAChunkBytes);
                        tma_load_2d_pair(dst, &map_h, kc * kAK, row0, in_leader(&sm.a_full[kc]));
                    } else {
                        mbar_arrive_expect_tx(&sm.a_full[kc], kAChunkBytes);
                        tma_load_2d(dst, &map_h, kc * kAK, row0, &sm.a_full[kc]);
                    }
                    issued[kc] = true;
                    ipar[kc] = it & 1;
                }
            }
            // drain: every issued copy has landed before the CTA may exit
            if (leader) {
                for (int kc = 0; kc < g.kchunks; ++kc)
                    if (issued[kc]) mbar_wait_cluster(&sm.a_full[kc], ipar[kc], err, 17);
            }
        }
    } else if (warp >= kEpilogueWarp0) {
        // --------------------------------------------------------------- epilogue
        const int lane_base = 32 * (warp & 3);
        const int row = lane_base + lane;
        const JointArgs& a = P.a;
        const int Vf = a.V + a.n_dur;
        uint32_t q = 0;
        bool ok = true;
        for (int unit = unit0; ok && unit < nunits; unit += units_stride) {
            const int n = begin + (unit * kCta + (int)rank) * kBM + row;
            const bool valid = n < end;
            int y = -1;
            int dn = 0;  // forward: the node's place in its utterance's diagonal-major weight block
            if (valid) {
                const NodeCoord c = node_coord(a.m, a.B, n);
                y = (c.u < c.Ub - 1) ? __ldg(a.targets + (int64_t)c.b * a.S + c.u) : -1;
                if (!kBwd) dn = __ldg(a.m.off + c.b) + diag_index(c.t, c.u, __ldg(a.m.Tb + c.b), c.Ub);
            }
            // forward state
            float m = -INFINITY, s = 0.f, lb = 0.f, ly = 0.f;
            float dur[kMaxDurCols];
#pragma unroll
            for (int k = 0; k < kMaxDurCols; ++k) dur[k] = 0.f;
            // backward per-node coefficients; rows past the pass end keep zeros, so
            // their G row is exp(0 - 0) * 0 = 0 (their A row, hence logits, is zero)
            float lse2 = 0.f, cb = 0.f, ct = 0.f, Pn = 0.f;  // lse2 = lse * log2(e)
            if (kBwd && valid) {
                lse2 = P.bwd.lse[n] * kLog2e;
                cb = P.bwd.cb[n];
                ct = P.bwd.ct[n];
                Pn = cb + ct;
#pragma unroll
                for (int k = 0; k < kMaxDurCols; ++k)  // duration-logit grads, used by the last chunk
                    if (k < a.n_dur) dur[k] = P.bwd.gdur[(int64_t)n * a.n_dur + k];
            }
            for (int j = 0; j < g.nchunks; ++j, ++q) {
                int col, width;
                chunk_of(g, j, col, width);
                const uint32_t buf = q & 1;
                if (!__all_sync(0xffffffffu, mbar_wait_cluster(&sm.t_full[buf], (q >> 1) & 1, err, 8))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t taddr = tmem_base + ((uint32_t)lane_base << 16) + buf * kNC;
                if constexpr (kStash) {
                    // Two sweeps of the chunk: its largest token logit mc, then the
                    // exp-sum relative to mc, the blank / label / duration gathers and
                    // the stash row x = logit - mc (nodes below stash.nodes).
                    const bool keep = valid && n < P.stash.nodes;
                    const int ng = width / 16;
                    float mc = -INFINITY;
                    for (int gi = 0; gi < ng; gi += 2) {
                        const int c0 = col + gi * 16;
                        if (gi + 1 < ng) {
                            float v[32];
                            tmem_ld32(taddr + gi * 16, v);
                            if (c0 + 32 <= a.V) {
#pragma unroll
                                for (int s2 = 1; s2 < 32; s2 *= 2)
#pragma unroll
                                    for (int i = 0; i + s2 < 32; i += 2 * s2) v[i] = fmaxf(v[i], v[i + s2]);
                                mc = fmaxf(mc, v[0]);
                            } else {
#pragma unroll
                                for (int i = 0; i < 32; ++i)
                                    if (c0 + i < a.V) mc = fmaxf(mc, v[i]);
                            }
                        } else {
                            float v[16];
                            tmem_ld16(taddr + gi * 16, v);
#pragma unroll
                            for (int i = 0; i < 16; ++i)
                                if (c0 + i < a.V) mc = fmaxf(mc, v[i]);
                        }
                    }
                    float sc = 0.f;
                    for (int gi = 0; gi < ng; ++gi) {
                        const int c0 = col + gi * 16;
                        float v[16], x[16];
                        tmem_ld16(taddr + gi * 16, v);
#pragma unroll
                        for (int i = 0; i < 16; ++i) x[i] = v[i] - mc;
                        if (c0 + 16 <= a.V) {
                            float e[16];
#pragma unroll
                            for (int i = 0; i < 16; ++i) e[i] = ex2_fast(x[i] * kLog2e);
#pragma unroll
                            for (int s2 = 1; s2 < 16; s2 *= 2)
#pragma unroll
                                for (int i = 0; i + s2 < 16; i += 2 * s2) e[i] += e[i + s2];
                            sc += e[0];
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
                                    sc += ex2_fast(x[i] * kLog2e);
                                    if (c == a.blank) lb = v[i];
                                    if (c == y) ly = v[i];
                                } else if (c < Vf) {
#pragma unroll
                                    for (int k = 0; k < kMaxDurCols; ++k)
                                        if (c - a.V == k) dur[k] = v[i];
                                }
                            }
                        }
                        if (keep) {
                            const int64_t e0 = (int64_t)n * g.vpad + c0;
                            if (g.parts == 1) {
                                uint4 w0, w1;
                                w0.x = pack_f16(x[0], x[1]);
                                w0.y = pack_f16(x[2], x[3]);
                                w0.z = pack_f16(x[4], x[5]);
                                w0.w = pack_f16(x[6], x[7]);
                                w1.x = pack_f16(x[8], x[9]);
                                w1.y = pack_f16(x[10], x[11]);
                                w1.z = pack_f16(x[12], x[13]);
                                w1.w = pack_f16(x[14], x[15]);
                                st_global_32B(static_cast<__half*>(P.stash.data) + e0, w0, w1);
                            } else {
                                float* dst = static_cast<float*>(P.stash.data) + e0;
#pragma unroll
                                for (int h = 0; h < 2; ++h) {
                                    const uint4 lo = make_uint4(__float_as_uint(x[8 * h]), __float_as_uint(x[8 * h + 1]),
                                                                __float_as_uint(x[8 * h + 2]),
                                                                __float_as_uint(x[8 * h + 3]));
                                    const uint4 hi = make_uint4(
                                        __float_as_uint(x[8 * h + 4]), __float_as_uint(x[8 * h + 5]),
                                        __float_as_uint(x[8 * h + 6]), __float_as_uint(x[8 * h + 7]));
                                    st_global_32B(dst + 8 * h, lo, hi);
                                }
                            }
                        }
                    }
                    if (mc > m) {
                        s = s * __expf(m - mc) + sc;
                        m = mc;
                    } else if (mc > -INFINITY) {
                        s += sc * __expf(mc - m);
                    }
                    if (keep) P.stash.meta[(int64_t)n * (g.nchunks + 2) + j] = mc;
                } else
                for (int gi = 0; gi < width / 16; ++gi) {
                    if (!kBwd && gi + 1 < width / 16 && col + gi * 16 + 32 <= a.V) {
                        // two token groups at once: one TMEM wait, and the max and the
                        // sum of the online log-sum-exp as pairwise trees, so the chain
                        // of this lane-quarter's single warp is 5 deep instead of 31
                        const int c0 = col + gi * 16;
                        float v[32], t[32];
                        tmem_ld32(taddr + gi * 16, v);
#pragma unroll
                        for (int i = 0; i < 32; ++i) t[i] = v[i];
#pragma unroll
                        for (int s2 = 1; s2 < 32; s2 *= 2)
#pragma unroll
                            for (int i = 0; i + s2 < 32; i += 2 * s2) t[i] = fmaxf(t[i], t[i + s2]);
                        if (t[0] > m) {
                            s = (m == -INFINITY) ? 0.f : s * __expf(m - t[0]);
                            m = t[0];
                        }
#pragma unroll
                        for (int i = 0; i < 32; ++i) t[i] = __expf(v[i] - m);
#pragma unroll
                        for (int s2 = 1; s2 < 32; s2 *= 2)
#pragma unroll
                            for (int i = 0; i + s2 < 32; i += 2 * s2) t[i] += t[i + s2];
                        s += t[0];
#pragma unroll
                        for (int i = 0; i < 32; ++i) {
                            if (c0 + i == a.blank) lb = v[i];
                            if (c0 + i == y) ly = v[i];
                        }
                        ++gi;
                        continue;
                    }
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
                    } else {
                        // G = softmax * (cb + ct) - cb [blank] - ct [label]; duration grads
                        float gv[16];
                        if (c0 + 16 <= a.V) {  // token columns only: branch-free
                            const int db = a.blank - c0, dy = y - c0;
#pragma unroll
                            for (int i = 0; i < 16; ++i) {
                                float x = ex2_fast(fmaf(v[i], kLog2e, -lse2)) * Pn;
                                x = (i == db) ? x - cb : x;
                                gv[i] = (i == dy) ? x - ct : x;
                            }
                        } else {
#pragma unroll
                            for (int i = 0; i < 16; ++i) {
                                const int c = c0 + i;
                                float x = 0.f;
                                if (c < a.V) {
                                    x = ex2_fast(fmaf(v[i], kLog2e, -lse2)) * Pn;
                                    if (c == a.blank) x -= cb;
                                    if (c == y) x -= ct;
                                } else {
#pragma unroll
                                    for (int k = 0; k < kMaxDurCols; ++k)
                                        if (c - a.V == k && k < a.n_dur) x = dur[k];
                                }
                                gv[i] = x;
                            }
                        }
                        auto pack16 = [](const float (&x)[16], uint4& u0, uint4& u1) {
                            u0.x = pack_bf16(x[0], x[1]);
                            u0.y = pack_bf16(x[2], x[3]);
                            u0.z = pack_bf16(x[4], x[5]);
                            u0.w = pack_bf16(x[6], x[7]);
                            u1.x = pack_bf16(x[8], x[9]);
                            u1.y = pack_bf16(x[10], x[11]);
                            u1.z = pack_bf16(x[12], x[13]);
                            u1.w = pack_bf16(x[14], x[15]);
                        };
                        uint4 w0, w1;
                        // one 32-byte store (a whole sector): rows are gw * 2 bytes, a multiple
                        // of 32, and groups start on 16-column boundaries
                        __nv_bfloat16* grow = P.G + (int64_t)(n - base) * g.gw + c0;
                        if (g.parts == 1) {
                            pack16(gv, w0, w1);
                            st_global_32B(grow, w0, w1);
                        } else {  // split fp32: G rows [hi | hi | lo]
                            float gl[16];
#pragma unroll
                            for (int i = 0; i < 16; ++i) {
                                const float h = __bfloat162float(__float2bfloat16_rn(gv[i]));
                                gl[i] = gv[i] - h;
                                gv[i] = h;
                            }
                            pack16(gv, w0, w1);
                            st_global_32B(grow, w0, w1);
                            st_global_32B(grow + g.vpad, w0, w1);
                            pack16(gl, w0, w1);
                            st_global_32B(grow + 2 * g.vpad, w0, w1);
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    if (kCta == 2)
                        mbar_arrive_cluster(in_leader(&sm.t_empty[buf]));
                    else
                        mbar_arrive(&sm.t_empty[buf]);
                }
            }
            if (!kBwd && ok && valid) {
                const float l = m + __logf(s);
                P.fwd.lse[n] = l;
                if (kStash && n < P.stash.nodes) {
                    float* meta = P.stash.meta + (int64_t)n * (g.nchunks + 2) + g.nchunks;
                    meta[0] = l;
                    meta[1] = __int_as_float(y);
                }
                P.fwd.lpb[dn] = lb - l - a.sigma;
                P.fwd.lpy[dn] = y >= 0 ? ly - l - a.sigma : kNeg;
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
                        if (k < a.n_dur) P.fwd.lpd[(int64_t)dn * a.n_dur + k] = dur[k] - lz;
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (kCta == 2) {
        cluster_sync();  // no CTA leaves while its pair may still read its smem or signal it
        tc_fence_after();
        if (warp == 1) tmem_dealloc_pair(tmem_base, kTmemCols);
    } else {
        tc_fence_after();
        if (warp == 1) tmem_dealloc(tmem_base, kTmemCols);
    }
}

// [joint_W; joint_W_dur] -> bf16 (vpad, kpad), zero padded; optionally also the
// transpose (kpad, vpad) used as the K-major B operand of dH.
__global__ void prep_weights_kernel(const float* __restrict__ W, const float* __restrict__ Wd,
                                    const float* __restrict__ bias, int V, int n_dur, int d, int vpad, int kp,
                                    int parts, __nv_bfloat16* __restrict__ Wf, __nv_bfloat16* __restrict__ Wt) {
    const int64_t total = (int64_t)vpad * kp;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int r = (int)(i / kp), k = (int)(i % kp);
        float x = 0.f;
        if (k < d) {
            if (r < V)
                x = W[(int64_t)r * d + k];
            else if (r < V + n_dur)
                x = Wd[(int64_t)(r - V) * d + k];
        } else if (k == d && bias && r < V) {
            x = bias[r];  // CTC head: the weight of the ones column
        }
        const __nv_bfloat16 hi = __float2bfloat16_rn(x);
        if (parts == 1) {
            Wf[i] = hi;
            if (Wt) Wt[(int64_t)k * vpad + r] = hi;
        } else {  // split fp32: Wf rows [hi | hi | lo], Wt rows [hi | lo | hi]
            const __nv_bfloat16 lo = __float2bfloat16_rn(x - __bfloat162float(hi));
            __nv_bfloat16* wf = Wf + (int64_t)r * 3 * kp + k;
            wf[0] = hi;
            wf[kp] = hi;
            wf[2 * kp] = lo;
            if (Wt) {
                __nv_bfloat16* wt = Wt + (int64_t)k * 3 * vpad + r;
                wt[0] = hi;
                wt[vpad] = lo;
                wt[2 * vpad] = hi;
            }
        }
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

// 3-D view of a row-major (rows, cols) bf16 matrix whose columns split into
// blocks of 64 (cols % 64 == 0): dims (64, rows, cols / 64). A box of
// (64, box_rows, nblk) lands in shared memory as nblk consecutive 128-byte
// swizzled (box_rows x 64) tiles, i.e. nblk 2-D boxes in one copy.
bool make_map_blocks(CUtensorMap* map, const void* base, int rows, int cols, int box_rows, int nblk) {
    auto enc = tensor_map_encoder();
    if (!enc || cols % 64 != 0) return false;
    cuuint64_t dims[3] = {64, (cuuint64_t)rows, (cuuint64_t)(cols / 64)};
    cuuint64_t strides[2] = {(cuuint64_t)cols * 2, 128};
    cuuint32_t box[3] = {64, (cuuint32_t)box_rows, (cuuint32_t)nblk};
    cuuint32_t estr[3] = {1, 1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

size_t al256(size_t x) { return (x + 255) & ~size_t(255); }

int dyn_smem_limit() {
    int dev = 0, v = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    return v;
}

// ------------------------------------------------------------------ passes
//
// Both directions run over passes of at most kMaxPassNodes nodes (or the
// ASR_B200_BWD_PASS_NODES override: a tuning knob, small values exercise
// multi-pass runs), so the per-pass bf16 buffers (H, and G in the backward)
// stay bounded whatever the batch.
constexpr int64_t kMaxPassNodes = 4 << 20;
constexpr int kPassAlign = 256;  // pass rows are padded to whole 256-row tiles

int64_t pass_nodes_limit() {
    const char* env = std::getenv("ASR_B200_BWD_PASS_NODES");
    if (env) {
        const long long v = std::atoll(env);
        if (v > 0) return v;
    }
    return kMaxPassNodes;
}

struct PassPlan {
    int64_t step;  // nodes per pass (multiple of kPassAlign) = rows of the per-pass buffers
    int passes;
};

PassPlan pass_plan(int64_t cap) {
    PassPlan pp;
    const int64_t want = std::max<int64_t>(1, std::min<int64_t>(cap, pass_nodes_limit()));
    pp.step = (want + kPassAlign - 1) / kPassAlign * kPassAlign;
    pp.passes = (int)std::max<int64_t>(1, (cap + pp.step - 1) / pp.step);
    return pp;
}

// bounds[p] = first node of pass p (p = 0..P), clamped to the node count.
__global__ void plan_passes_kernel(LatticeMeta m, int B, int P, int64_t step, int32_t* __restrict__ bounds) {
    const int p = blockIdx.x * blockDim.x + threadIdx.x;
    if (p > P) return;
    const int N = total_nodes(m, B);
    bounds[p] = (p == P) ? N : (int)std::min<int64_t>((int64_t)p * step, N);
}

// H[r, k] = bf16(tanh(enc[b, t, k] + dec[b, u, k])) for the pass's node r (row
// r = node - pass start, k < kpad, zero for k >= d). Rows from the pass end up
// to the next 256-row boundary are zeroed: the joint kernels read whole tiles.
// Bound by the H writes (1280 B per node at d = 640) and by the MUFU pipe (one
// tanh per element plus one bf16 pack per pair).
//
// Scalar path (d % 8 != 0 or unaligned rows): each warp walks a run of
// kHiddenRun consecutive rows (one coordinate search per run, then (t, u)
// increments), element loads, 16-byte stores.
constexpr int kHiddenRun = 64;

__device__ __forceinline__ float load1(const float* p) { return __ldg(p); }
__device__ __forceinline__ float load1(const __nv_bfloat16* p) { return __bfloat162float(p[0]); }

// H element: tanh.approx for the bf16 path (below bf16 resolution); the
// accurate tanhf for the split fp32 path, whose parts resolve ~2^-16.
template <int PARTS>
__device__ __forceinline__ float hidden_tanh(float x) {
    return PARTS == 1 ? tanh_fast(x) : tanhf(x);
}

__device__ __forceinline__ void store_h(__nv_bfloat16* p, const float (&h)[4]) {
    *reinterpret_cast<uint2*>(p) = make_uint2(pack_bf16(h[0], h[1]), pack_bf16(h[2], h[3]));
}
__device__ __forceinline__ void store_h(__nv_bfloat16* p, const float (&h)[8]) {
    *reinterpret_cast<uint4*>(p) =
        make_uint4(pack_bf16(h[0], h[1]), pack_bf16(h[2], h[3]), pack_bf16(h[4], h[5]), pack_bf16(h[6], h[7]));
}

// Stores CE columns of an H row: bf16(h), or for the split path the parts
// [hi | lo | hi] at column offsets 0, kp and 2 kp.
template <int PARTS, int CE>
__device__ __forceinline__ void store_parts(__nv_bfloat16* p, const float (&h)[CE], int kp) {
    if (PARTS == 1) {
        store_h(p, h);
        return;
    }
    float hi[CE], lo[CE];
#pragma unroll
    for (int i = 0; i < CE; ++i) {
        hi[i] = __bfloat162float(__float2bfloat16_rn(h[i]));
        lo[i] = h[i] - hi[i];
    }
    store_h(p, hi);
    store_h(p + kp, lo);
    store_h(p + 2 * kp, hi);
}

template <typename TA, int PARTS>
__global__ void __launch_bounds__(256, 3) hidden_kernel(LatticeMeta m, int B, const TA* __restrict__ enc,
                                                        const TA* __restrict__ dec, int T, int U, int d, int kp,
                                                        const int32_t* __restrict__ bounds, int pass,
                                                        __nv_bfloat16* __restrict__ H) {
    const int N = total_nodes(m, B);
    const int s = min(bounds[pass], N), e = min(bounds[pass + 1], N);
    const int rows = e - s;
    const int rows_pad = (rows + kPassAlign - 1) / kPassAlign * kPassAlign;
    const int c8n = kp / 8;
    const int64_t stride = (int64_t)PARTS * kp;
    const int lane = threadIdx.x & 31;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    for (int r0 = ((blockIdx.x * blockDim.x + threadIdx.x) >> 5) * kHiddenRun; r0 < rows_pad;
         r0 += nwarps * kHiddenRun) {
        const int r1 = min(r0 + kHiddenRun, rows_pad);
        NodeCoord c{};
        int Tb = 0;
        if (r0 < rows) {
            c = node_coord(m, B, s + r0);
            Tb = __ldg(m.Tb + c.b);
        }
        for (int r = r0; r < r1; ++r) {
            __nv_bfloat16* dst = H + (int64_t)r * stride;
            if (r >= rows) {
                const float z[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
                for (int k8 = lane; k8 < c8n; k8 += 32) store_parts<PARTS, 8>(dst + k8 * 8, z, kp);
                continue;
            }
            const TA* er = enc + ((int64_t)c.b * T + c.t) * d;
            const TA* dr = dec + ((int64_t)c.b * U + c.u) * d;
            for (int k8 = lane; k8 < c8n; k8 += 32) {
                const int k = k8 * 8;
                float h[8];
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    h[i] = k + i < d ? hidden_tanh<PARTS>(load1(er + k + i) + load1(dr + k + i)) : 0.f;
                store_parts<PARTS, 8>(dst + k, h, kp);
            }
            // next node: next label position, next frame, or the next utterance
            if (++c.u == c.Ub) {
                c.u = 0;
                if (++c.t == Tb && r + 1 < rows) {
                    c = node_coord(m, B, s + r + 1);
                    Tb = __ldg(m.Tb + c.b);
                }
            }
        }
    }
}

// Vector path of the hidden rows (d % 8 == 0, 16-byte aligned rows). Each warp
// takes a run of kFlatRun rows: lane i resolves row i's enc and dec row indices
// once into shared memory, then the warp walks the run's rows x column chunks
// as one flat index space. A chunk is the 16 bytes of input one lane loads from
// each of enc and dec (4 fp32 or 8 bf16 columns), so every warp load covers 512
// contiguous bytes (no sector is fetched half used) and no lane idles on a
// partial column group. UNR chunks per lane are in flight at a time, all their
// loads issued before the first tanh.
constexpr int kFlatRun = 32;
constexpr int kFlatWarps = 8;

template <typename TA>
struct Chunk;
template <>
struct Chunk<float> {  // 4 columns; 8 bytes of H
    static constexpr int kCols = 4;
    float4 v;
    __device__ __forceinline__ void load(const float* __restrict__ p) { v = __ldg(reinterpret_cast<const float4*>(p)); }
    __device__ __forceinline__ void get(float (&x)[kCols]) const { x[0] = v.x, x[1] = v.y, x[2] = v.z, x[3] = v.w; }
};
template <>
struct Chunk<__nv_bfloat16> {  // 8 columns; 16 bytes of H
    static constexpr int kCols = 8;
    uint4 v;
    __device__ __forceinline__ void load(const __nv_bfloat16* __restrict__ p) {
        v = __ldg(reinterpret_cast<const uint4*>(p));
    }
    __device__ __forceinline__ void get(float (&x)[kCols]) const {
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __bfloat1622float2(h[i]);
            x[2 * i] = f.x, x[2 * i + 1] = f.y;
        }
    }
};

template <int UNR>
constexpr int kFlatMinBlocks = UNR <= 4 ? 3 : 2;

template <typename TA, int UNR, int PARTS>
__global__ void __launch_bounds__(kFlatWarps * 32, kFlatMinBlocks<UNR>)
    hidden_flat_kernel(LatticeMeta m, int B, const TA* __restrict__ enc, const TA* __restrict__ dec, int T, int U,
                       int d, int kp, const int32_t* __restrict__ bounds, int pass, __nv_bfloat16* __restrict__ H) {
    constexpr int CE = Chunk<TA>::kCols;
    __shared__ int2 rows_sm[kFlatWarps][kFlatRun];
    const int N = total_nodes(m, B);
    const int s = min(bounds[pass], N), e = min(bounds[pass + 1], N);
    const int rows = e - s;
    const int rows_pad = (rows + kPassAlign - 1) / kPassAlign * kPassAlign;  // a multiple of kFlatRun
    const int cn = kp / CE, cd = d / CE;  // chunks per H row (one part), chunks holding columns < d
    const int64_t stride = (int64_t)PARTS * kp;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int nwarps = gridDim.x * kFlatWarps;
    int2* rs = rows_sm[w];
    const int total = kFlatRun * cn;  // chunks per run
    for (int r0 = (blockIdx.x * kFlatWarps + w) * kFlatRun; r0 < rows_pad; r0 += nwarps * kFlatRun) {
        {
            const int r = r0 + lane;
            int2 v = make_int2(-1, -1);  // padding row: zeros
            if (r < rows) {
                const NodeCoord c = node_coord(m, B, s + r);
                v = make_int2(c.b * T + c.t, c.b * U + c.u);
            }
            rs[lane] = v;
        }
        __syncwarp();
        __nv_bfloat16* dst = H + (int64_t)r0 * stride;
        int rr = 0, kc = lane;  // chunk q = lane + 32 i lies in row rr, column chunk kc
        while (kc >= cn) kc -= cn, ++rr;
        for (int q0 = 0; q0 < total; q0 += 32 * UNR) {
            Chunk<TA> ev[UNR], dv[UNR];
            int rj[UNR], kj[UNR];
#pragma unroll
            for (int j = 0; j < UNR; ++j) {
                rj[j] = rr, kj[j] = kc;
                const int2 v = rr < kFlatRun ? rs[rr] : make_int2(-1, -1);
                if (v.x >= 0 && kc < cd) {
                    ev[j].load(enc + (int64_t)v.x * d + kc * CE);
                    dv[j].load(dec + (int64_t)v.y * d + kc * CE);
                } else {
                    kj[j] = -1 - kc;  // zero chunk (padding row or column)
                }
                kc += 32;
                while (kc >= cn) kc -= cn, ++rr;
            }
#pragma unroll
            for (int j = 0; j < UNR; ++j) {
                if (rj[j] >= kFlatRun) break;
                float h[CE];
                int k = kj[j];
                if (k >= 0) {
                    float x[CE], y[CE];
                    ev[j].get(x);
                    dv[j].get(y);
#pragma unroll
                    for (int i = 0; i < CE; ++i) h[i] = hidden_tanh<PARTS>(x[i] + y[i]);
                } else {
                    k = -1 - k;
#pragma unroll
                    for (int i = 0; i < CE; ++i) h[i] = 0.f;
                }
                store_parts<PARTS, CE>(dst + (int64_t)rj[j] * stride + k * CE, h, kp);
            }
        }
        __syncwarp();  // rs is rewritten by the next run
    }
}

// Row-stationary vector path for rows of at most 32 * 8 chunks (kpad <= 1024 for
// fp32 activations, 2048 for bf16): lane l owns chunks l, l + 32, ..., l + 32 (J-1)
// of every row, so the column offsets and their validity are fixed per lane and
// a row costs one shared-memory descriptor read and a base address. Rows are
// taken in groups of up to R consecutive rows of one frame: the group's R dec
// rows are loaded together, and the frame's enc row is loaded only when the
// frame changes and otherwise stays in registers, so the L1 data path carries
// one input row per H row instead of two. Same run and descriptor scheme as the
// flat kernel above.
template <typename TA, int J, int R>
constexpr int kRowsMinBlocks = (R + 1) * J * 4 <= 40 ? 3 : 2;

template <typename TA, int J, int R, int PARTS>
__global__ void __launch_bounds__(kFlatWarps * 32, (kRowsMinBlocks<TA, J, R>))
    hidden_rows_kernel(LatticeMeta m, int B, const TA* __restrict__ enc, const TA* __restrict__ dec, int T, int U,
                       int d, int kp, const int32_t* __restrict__ bounds, int pass, __nv_bfloat16* __restrict__ H) {
    constexpr int CE = Chunk<TA>::kCols;
    __shared__ int2 rows_sm[kFlatWarps][kFlatRun + 1];
    const int N = total_nodes(m, B);
    const int s = min(bounds[pass], N), e = min(bounds[pass + 1], N);
    const int rows = e - s;
    const int rows_pad = (rows + kPassAlign - 1) / kPassAlign * kPassAlign;
    const int cn = kp / CE, cd = d / CE;
    const int64_t stride = (int64_t)PARTS * kp;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int nwarps = gridDim.x * kFlatWarps;
    int2* rs = rows_sm[w];
    if (lane == 0) rs[kFlatRun] = make_int2(-2, -2);  // sentinel: ends every frame group
    for (int r0 = (blockIdx.x * kFlatWarps + w) * kFlatRun; r0 < rows_pad; r0 += nwarps * kFlatRun) {
        {
            const int r = r0 + lane;
            int2 v = make_int2(-1, -1);  // padding row: zeros
            if (r < rows) {
                const NodeCoord c = node_coord(m, B, s + r);
                v = make_int2(c.b * T + c.t, c.b * U + c.u);
            }
            rs[lane] = v;
        }
        __syncwarp();
        Chunk<TA> ev[J];
        int ecur = -1;  // enc row held in ev (-1: none)
        int rr = 0;
#pragma unroll 1
        while (rr < kFlatRun) {
            const int erow = rs[rr].x;  // warp-uniform
            int drow[R];
            int n = 0;  // rows of this group: consecutive rows of frame erow, at most R
#pragma unroll
            for (int i = 0; i < R; ++i) {
                const int2 v = rs[rr + i < kFlatRun ? rr + i : kFlatRun];
                drow[i] = v.y;
                if (n == i && v.x == erow) n = i + 1;
            }
            Chunk<TA> dv[R][J];
            if (erow >= 0) {
#pragma unroll
                for (int i = 0; i < R; ++i) {
                    if (i < n) {
                        const TA* db = dec + (int64_t)drow[i] * d + lane * CE;
#pragma unroll
                        for (int j = 0; j < J; ++j)
                            if (lane + 32 * j < cd) dv[i][j].load(db + 32 * CE * j);
                    }
                }
                if (erow != ecur) {
                    const TA* eb = enc + (int64_t)erow * d + lane * CE;
#pragma unroll
                    for (int j = 0; j < J; ++j)
                        if (lane + 32 * j < cd) ev[j].load(eb + 32 * CE * j);
                    ecur = erow;
                }
            }
#pragma unroll
            for (int i = 0; i < R; ++i) {
                if (i >= n) break;
                __nv_bfloat16* out = H + (int64_t)(r0 + rr + i) * stride + lane * CE;
#pragma unroll
                for (int j = 0; j < J; ++j) {
                    if (lane + 32 * j >= cn) break;
                    float h[CE];
                    if (erow >= 0 && lane + 32 * j < cd) {
                        float x[CE], y[CE];
                        ev[j].get(x);
                        dv[i][j].get(y);
#pragma unroll
                        for (int k = 0; k < CE; ++k) h[k] = hidden_tanh<PARTS>(x[k] + y[k]);
                    } else {
#pragma unroll
                        for (int k = 0; k < CE; ++k) h[k] = 0.f;
                    }
                    store_parts<PARTS, CE>(out + 32 * CE * j, h, kp);
                }
            }
            rr += n;
        }
        __syncwarp();  // rs is rewritten by the next run
    }
}

template <typename TA, int J, int R, int PARTS>
void launch_rows(const JointArgs& a, const TA* enc, const TA* dec, int kp, const int32_t* bounds, int pass,
                 __nv_bfloat16* H, cudaStream_t st) {
    hidden_rows_kernel<TA, J, R, PARTS><<<sm_count() * kRowsMinBlocks<TA, J, R>, kFlatWarps * 32, 0, st>>>(
        a.m, a.B, enc, dec, a.T, a.U, a.d, kp, bounds, pass, H);
}

// J = chunks per lane per row (1..8). Three rows in flight per warp where the
// registers allow it (measured best on B200 for d = 640 in both activation
// types), two for the widest rows.
template <typename TA, int PARTS>
bool launch_rows_j(int J, const JointArgs& a, const TA* enc, const TA* dec, int kp, const int32_t* bounds, int pass,
                   __nv_bfloat16* H, cudaStream_t st) {
    switch (J) {
        case 1: launch_rows<TA, 1, 3, PARTS>(a, enc, dec, kp, bounds, pass, H, st); return true;
        case 2: launch_rows<TA, 2, 3, PARTS>(a, enc, dec, kp, bounds, pass, H, st); return true;
        case 3: launch_rows<TA, 3, 3, PARTS>(a, enc, dec, kp, bounds, pass, H, st); return true;
        case 4: launch_rows<TA, 4, 3, PARTS>(a, enc, dec, kp, bounds, pass, H, st); return true;
        case 5: launch_rows<TA, 5, 3, PARTS>(a, enc, dec, kp, bounds, pass, H, st); return true;
        case 6: launch_rows<TA, 6, 2, PARTS>(a, enc, dec, kp, bounds, pass, H, st); return true;
        case 7: launch_rows<TA, 7, 2, PARTS>(a, enc, dec, kp, bounds, pass, H, st); return true;
        case 8: launch_rows<TA, 8, 2, PARTS>(a, enc, dec, kp, bounds, pass, H, st); return true;
        default: return false;
    }
}

template <typename TA, int UNR, int PARTS>
void launch_flat(const JointArgs& a, const TA* enc, const TA* dec, int kp, const int32_t* bounds, int pass,
                 __nv_bfloat16* H, cudaStream_t st) {
    hidden_flat_kernel<TA, UNR, PARTS><<<sm_count() * kFlatMinBlocks<UNR>, kFlatWarps * 32, 0, st>>>(
        a.m, a.B, enc, dec, a.T, a.U, a.d, kp, bounds, pass, H);
}

// CTC head hidden rows: one warp per frame row, H = bf16(x * rsqrt(mean(x^2) + eps)
// * g) (torch's rms_norm: fp32 statistics, the result rounded to bf16 as the
// autocast Linear rounds its input), then a ones column at k = d when the head has
// a bias; columns past it and rows up to the next 256-row boundary are zero.
template <typename TA>
__global__ void __launch_bounds__(256) rms_hidden_kernel(LatticeMeta m, int B, const TA* __restrict__ enc,
                                                         const float* __restrict__ g, float eps, int ones, int T,
                                                         int d, int kpad, const int32_t* __restrict__ bounds, int pass,
                                                         __nv_bfloat16* __restrict__ H) {
    const int N = total_nodes(m, B);
    const int s = min(bounds[pass], N), e = min(bounds[pass + 1], N);
    const int rows = e - s;
    const int rows_pad = (rows + kPassAlign - 1) / kPassAlign * kPassAlign;
    const int lane = threadIdx.x & 31;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    for (int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows_pad; r += nwarps) {
        __nv_bfloat16* dst = H + (int64_t)r * kpad;
        if (r >= rows) {
            for (int k = lane; k < kpad; k += 32) dst[k] = __float2bfloat16_rn(0.f);
            continue;
        }
        const NodeCoord c = node_coord(m, B, s + r);  // U_b = 1: node = frame
        const TA* x = enc + ((int64_t)c.b * T + c.t) * d;
        float ss = 0.f;
        for (int k = lane; k < d; k += 32) {
            const float v = load1(x + k);
            ss = fmaf(v, v, ss);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float rstd = rsqrtf(ss / (float)d + eps);
        for (int k = lane; k < kpad; k += 32) {
            float h = 0.f;
            if (k < d)
                h = load1(x + k) * rstd * __ldg(g + k);
            else if (k == d && ones)
                h = 1.f;
            dst[k] = __float2bfloat16_rn(h);
        }
    }
}

template <int PARTS>
void launch_hidden_parts(const JointArgs& a, int kp, const int32_t* bounds, int pass, __nv_bfloat16* H,
                         cudaStream_t st) {
    if (a.vec) {
        // row-stationary kernel up to 8 chunks per lane, the flat kernel for wider rows
        const int J = (kp / (a.enc16 ? 8 : 4) + 31) / 32;
        if (a.enc16) {
            if (!launch_rows_j<__nv_bfloat16, PARTS>(J, a, a.enc16, a.dec16, kp, bounds, pass, H, st))
                launch_flat<__nv_bfloat16, 4, PARTS>(a, a.enc16, a.dec16, kp, bounds, pass, H, st);
        } else {
            if (!launch_rows_j<float, PARTS>(J, a, a.enc, a.dec, kp, bounds, pass, H, st))
                launch_flat<float, 4, PARTS>(a, a.enc, a.dec, kp, bounds, pass, H, st);
        }
    } else if (a.enc16) {
        hidden_kernel<__nv_bfloat16, PARTS><<<sm_count() * 8, 256, 0, st>>>(a.m, a.B, a.enc16, a.dec16, a.T, a.U,
                                                                            a.d, kp, bounds, pass, H);
    } else {
        hidden_kernel<float, PARTS><<<sm_count() * 8, 256, 0, st>>>(a.m, a.B, a.enc, a.dec, a.T, a.U, a.d, kp, bounds,
                                                                    pass, H);
    }
}

// The hidden rows of one pass: H = bf16(tanh(enc + dec)) (g.kpad columns), or
// its split parts, or the CTC head's RMSNorm rows.
int launch_hidden(const JointArgs& a, const Geom& g, const int32_t* bounds, int pass, __nv_bfloat16* H,
                  cudaStream_t st) {
    KernelTimer kt("joint_hidden", st);
    if (a.head) {
        if (a.enc16)
            rms_hidden_kernel<__nv_bfloat16><<<sm_count() * 8, 256, 0, st>>>(
                a.m, a.B, a.enc16, a.rms_g, a.rms_eps, a.bias ? 1 : 0, a.T, a.d, g.kpad, bounds, pass, H);
        else
            rms_hidden_kernel<float><<<sm_count() * 8, 256, 0, st>>>(a.m, a.B, a.enc, a.rms_g, a.rms_eps,
                                                                     a.bias ? 1 : 0, a.T, a.d, g.kpad, bounds, pass, H);
        ASR_LAUNCH_CHECK();
        return ASR_OK;
    }
    if (g.parts == 3)
        launch_hidden_parts<3>(a, g.kp, bounds, pass, H, st);
    else
        launch_hidden_parts<1>(a, g.kp, bounds, pass, H, st);
    ASR_LAUNCH_CHECK();
    return ASR_OK;
}

// CTA pairs (cta_group::2) for the joint kernel when ASR_B200_JOINT_PAIRS=1. Off
// by default: on B200 the single-CTA kernel measured faster (5.9 vs 7.1 ms for
// the config-5-like B = 128 forward), the pair paying cross-CTA barrier traffic
// for a weight stream that the 128-byte stages already keep up with.
bool joint_pairs() {
    static const bool pairs = [] {
        const char* e = std::getenv("ASR_B200_JOINT_PAIRS");
        return e && e[0] == '1';
    }();
    return pairs;
}

// Streamed hidden tiles: the default (see kStreamStagesMax); required above
// 64 * kMaxKChunks hidden columns. ASR_B200_JOINT_STREAM=0, or CTA pairs (which
// split the resident tile's MMA across two SMs), keep the hidden tile resident.
bool joint_stream(const Geom& g) {
    if (g.kchunks > kMaxKChunks) return true;
    static const int force = [] {
        const char* e = std::getenv("ASR_B200_JOINT_STREAM");
        return e ? (e[0] == '1' ? 1 : 0) : -1;
    }();
    if (force == 0) return false;
    return force == 1 || !joint_pairs();
}

// Weight tensor maps of the joint kernel: a regular chunk and the last chunk,
// each split across the pair when pairs are used.
bool joint_weight_maps(const Geom& g, const __nv_bfloat16* Wf, bool pairs, CUtensorMap* mfull, CUtensorMap* mtail) {
    const int split = pairs ? 2 : 1;
    return make_map(mfull, Wf, g.vpad, g.kpad, kBK, g.cw / split, CU_TENSOR_MAP_SWIZZLE_128B) &&
           make_map(mtail, Wf, g.vpad, g.kpad, kBK, g.lw / split, CU_TENSOR_MAP_SWIZZLE_128B);
}

// Persistent launch over `tiles` 128-node tiles (at most one CTA per SM).
template <bool kBwd, bool kStash = false>
int launch_joint(bool pairs, int64_t tiles, size_t smem, const CUtensorMap& mfull, const CUtensorMap& mtail,
                 const CUtensorMap& mh, const TcParams& P, cudaStream_t st) {
    const int sms = sm_count();
    const int grid1 = (int)std::max<int64_t>(1, std::min<int64_t>(tiles, sms));
    if (joint_stream(P.g)) {  // streamed hidden tiles
        const size_t smem_s = smem_bytes_for(P.g.kchunks, true, P.g.sstage, P.g.nstream);
        auto kern = tc_joint_kernel<kBwd, 1, true, kStash>;
        ASR_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_s));
        kern<<<grid1, kThreads, smem_s, st>>>(mfull, mtail, mh, P);
        ASR_LAUNCH_CHECK();
        return ASR_OK;
    }
    if (!pairs || kStash) {
        auto kern = tc_joint_kernel<kBwd, 1, false, kStash>;
        ASR_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        kern<<<grid1, kThreads, smem, st>>>(mfull, mtail, mh, P);
        ASR_LAUNCH_CHECK();
        return ASR_OK;
    }
    ASR_CUDA_TRY(cudaFuncSetAttribute(tc_joint_kernel<kBwd, 2, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)smem));
    const int64_t units = (tiles + 1) / 2;
    const int clusters = (int)std::max<int64_t>(1, std::min<int64_t>(units, sms / 2));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * clusters);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    ASR_CUDA_TRY(cudaLaunchKernelEx(&cfg, tc_joint_kernel<kBwd, 2, false>, mfull, mtail, mh, P));
    return ASR_OK;
}

}  // namespace

// Hidden dimensions up to 64 * kMaxKChunks keep the hidden tile resident; larger
// ones (up to 4096) stream it.
constexpr int kMaxStreamKChunks = 64;

bool tc_supported(const JointArgs& a) {
    const Geom g = make_geom(a);
    const bool stream = g.kchunks > kMaxKChunks;
    return g.kchunks <= kMaxStreamKChunks && a.n_dur <= kMaxDurCols && tensor_map_encoder() != nullptr &&
           (int)smem_bytes_for(g.kchunks, stream, g.sstage, g.nstream) <= dyn_smem_limit();
}

// Forward scratch: bf16 weights, the per-pass hidden rows, pass bounds, error word.
struct FwdLayout {
    PassPlan pp;
    size_t wf, h, bounds, err, total;
};

FwdLayout fwd_layout(const JointArgs& a, int64_t cap) {
    const Geom g = make_geom(a);
    FwdLayout L;
    L.pp = pass_plan(cap);
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t o = off;
        off += al256(bytes);
        return o;
    };
    L.wf = take(sizeof(__nv_bfloat16) * (size_t)g.vpad * g.kpad);
    L.h = take(sizeof(__nv_bfloat16) * (size_t)L.pp.step * g.kpad);
    L.bounds = take(sizeof(int32_t) * (L.pp.passes + 1));
    L.err = take(sizeof(int));
    L.total = off;
    return L;
}

size_t tc_forward_scratch_bytes(const JointArgs& a, int node_capacity) {
    return fwd_layout(a, node_capacity).total + 256;
}

// Stashed node counts are whole 256-node tiles of the d_hidden kernel, so the
// recompute kernel's tiles after the stash start on a tile of the pass.
constexpr int kStashAlign = 256;
constexpr int kStashMaxChunks = 16;  // vocabulary chunks of a stashed row (vpad <= 16 x 256)

size_t tc_stash_bytes_per_node(const JointArgs& a) {
    const Geom g = make_geom(a);
    return (size_t)g.vpad * (g.parts == 1 ? sizeof(__half) : sizeof(float)) + sizeof(float) * (g.nchunks + 2);
}

LogitStash tc_stash_carve(const JointArgs& a, void* stash, size_t bytes) {
    LogitStash s{nullptr, nullptr, 0};
    const size_t per = tc_stash_bytes_per_node(a);
    if (!stash || bytes <= 512 || make_geom(a).nchunks > kStashMaxChunks) return s;
    const int64_t nodes = std::min<int64_t>((int64_t)((bytes - 512) / per) / kStashAlign * kStashAlign, INT32_MAX / 2);
    if (nodes <= 0) return s;
    const Geom g = make_geom(a);
    char* p = reinterpret_cast<char*>(al256(reinterpret_cast<uintptr_t>(stash)));
    s.data = p;
    p += al256((size_t)nodes * g.vpad * (g.parts == 1 ? sizeof(__half) : sizeof(float)));
    s.meta = reinterpret_cast<float*>(p);
    s.nodes = (int)nodes;
    return s;
}

int tc_joint_forward(const JointArgs& a, const JointFwdOut& o, int node_capacity, void* scratch, size_t scratch_bytes,
                     cudaStream_t st, const LogitStash& stash) {
    const Geom g = make_geom(a);
    const FwdLayout L = fwd_layout(a, node_capacity);
    if (scratch_bytes < L.total) return ASR_ERR_WORKSPACE;
    char* base = reinterpret_cast<char*>(scratch);
    auto* Wf = reinterpret_cast<__nv_bfloat16*>(base + L.wf);
    auto* H = reinterpret_cast<__nv_bfloat16*>(base + L.h);
    auto* bounds = reinterpret_cast<int32_t*>(base + L.bounds);
    int* err = reinterpret_cast<int*>(base + L.err);
    ASR_CUDA_TRY(cudaMemsetAsync(err, 0, sizeof(int), st));
    {
        KernelTimer kt("joint_prep_weights", st);
        prep_weights_kernel<<<sm_count() * 4, 256, 0, st>>>(a.W, a.Wd, a.head ? a.bias : nullptr, a.V, a.n_dur,
                                                             a.d, g.vpad, g.kp, g.parts, Wf, nullptr);
        ASR_LAUNCH_CHECK();
        plan_passes_kernel<<<(L.pp.passes + 1 + 127) / 128, 128, 0, st>>>(a.m, a.B, L.pp.passes, L.pp.step, bounds);
        ASR_LAUNCH_CHECK();
    }
    const bool use_stash = stash.nodes > 0 && !a.head;
    // pairs use the resident hidden tile; the stash-writing forward runs single CTAs
    const bool pairs = joint_pairs() && !joint_stream(g) && !use_stash;
    CUtensorMap mfull, mtail, mh;
    if (!joint_weight_maps(g, Wf, pairs, &mfull, &mtail)) return ASR_ERR_CUDA;
    if (!make_map(&mh, H, (int)L.pp.step, g.kpad, kAK, kBM, CU_TENSOR_MAP_SWIZZLE_128B)) return ASR_ERR_CUDA;
    TcParams P;
    std::memset(&P, 0, sizeof(P));
    P.a = a;
    P.g = g;
    P.fwd = o;
    P.range.bounds = bounds;
    if (use_stash) P.stash = stash;
    P.err = err;
    for (int p = 0; p < L.pp.passes; ++p) {
        P.range.pass = p;
        int rc = launch_hidden(a, g, bounds, p, H, st);
        if (rc != ASR_OK) return rc;
        KernelTimer kt("joint_fwd_tc", st);
        rc = use_stash
                 ? launch_joint<false, true>(pairs, L.pp.step / kBM, smem_bytes_for(g.kchunks), mfull, mtail, mh, P, st)
                 : launch_joint<false>(pairs, L.pp.step / kBM, smem_bytes_for(g.kchunks), mfull, mtail, mh, P, st);
        if (rc != ASR_OK) return rc;
    }
    return ASR_OK;
}

// ------------------------------------------------------ dlogits from the stash
//
// G rows of the stashed nodes of a pass, [base, min(end, stash.nodes)):
//   G[n, c] = exp(x[n, c] + ref[n, j] - lse[n]) * (cb + ct) - cb [c = blank] - ct [c = label]
// for token columns (x the stashed logit - ref, j = c / cw), the duration-logit
// gradients for the duration columns, zero for the padding; the split fp32 mode
// stores the parts [hi | hi | lo]. A CTA takes tiles of kStashRows consecutive
// rows: their meta rows, posteriors and duration gradients (contiguous runs)
// go to shared memory first, then the tile's (row, 16-column group) items are
// walked flat with kBatch items' stash loads in flight per thread before the
// first G store (32-byte accesses, 1 KB contiguous per warp), so any vocabulary
// size keeps all lanes busy. The blank and label corrections are applied only
// to the items that hold those columns. Bound by HBM: the stash row read (2 B per column,
// 4 in the split mode) and the G row written. When the stash covers the rest of
// the pass, rows up to the next 128-row boundary are zeroed, as the recompute
// kernel's last tile does: the dW kernel reads whole 64-row blocks.

namespace {

struct StashParams {
    JointArgs a;
    Geom g;
    const int32_t* bounds;
    int pass;
    LogitStash stash;
    JointBwdIn in;
    __nv_bfloat16* G;
    uint32_t groups;       // 16-column groups of a row (vpad / 16)
    uint32_t magic_row;    // ceil(2^32 / groups): item / groups = umulhi(item, magic_row); 0: groups = 1
    uint32_t magic_chunk;  // ceil(2^32 / (cw / 16)): group -> vocabulary chunk; 0: cw = 16
};

constexpr int kStashRows = 128;  // rows per CTA tile

// item / groups (0 = divide by one: ceil(2^32 / 1) does not fit the multiplier)
__device__ __forceinline__ uint32_t row_of(uint32_t item, const StashParams& P) {
    return P.magic_row ? __umulhi(item, P.magic_row) : item;
}
constexpr int kStashThreads = 256;

template <int PARTS>
__global__ void __launch_bounds__(kStashThreads, 3) stash_dlogits_kernel(StashParams P) {
    // an item is 16 columns of a row: one or two 32-byte stash loads (fp16 / fp32)
    constexpr int kES = PARTS == 1 ? 2 : 4;      // bytes per stashed value
    constexpr int kLoads = PARTS == 1 ? 2 : 4;   // 16-byte loads per item
    constexpr int kBatch = PARTS == 1 ? 4 : 2;   // items whose stash loads are in flight together
    __shared__ float s_e[kStashRows * kStashMaxChunks];  // ref * log2(e) - lse * log2(e) per (row, chunk)
    __shared__ float s_cb[kStashRows], s_ct[kStashRows], s_pn[kStashRows];
    __shared__ int s_y[kStashRows];
    __shared__ float s_gd[kStashRows * kMaxDurCols];
    const JointArgs& a = P.a;
    const Geom& g = P.g;
    const int N = total_nodes(a.m, a.B);
    const int base = min(P.bounds[P.pass], N), end = min(P.bounds[P.pass + 1], N);
    const int split = min(end, max(base, P.stash.nodes));
    const int rows = split - base;
    const int zrows = (split == end ? (end - base + 127) / 128 * 128 : rows) - rows;
    const int nch = g.nchunks, mw = nch + 2, Vf = a.V + a.n_dur;
    const int ntiles = (rows + kStashRows - 1) / kStashRows;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
        const int r0 = tile * kStashRows;
        const int R = min(kStashRows, rows - r0);
        const int64_t row0 = (int64_t)(base + r0);  // global node of the tile's first row
        __syncthreads();  // the previous tile's coefficients are no longer read
        // every coefficient load of the row issued before the first shared store
        // (a load behind each store would pay one memory latency per value)
        if (threadIdx.x < R) {
            const int64_t n = row0 + threadIdx.x;
            const float* meta = P.stash.meta + n * mw;
            float ref[kStashMaxChunks];
#pragma unroll
            for (int j = 0; j < kStashMaxChunks; ++j) ref[j] = j < nch ? __ldg(meta + j) : 0.f;
            const float lse = __ldg(meta + nch), yv = __ldg(meta + nch + 1);
            const float cb = __ldg(P.in.cb + n), ct = __ldg(P.in.ct + n);
            float gd[kMaxDurCols];
#pragma unroll
            for (int k = 0; k < kMaxDurCols; ++k) gd[k] = k < a.n_dur ? __ldg(P.in.gdur + n * a.n_dur + k) : 0.f;
            const float l2 = lse * kLog2e;
#pragma unroll
            for (int j = 0; j < kStashMaxChunks; ++j)
                if (j < nch) s_e[threadIdx.x * kStashMaxChunks + j] = fmaf(ref[j], kLog2e, -l2);
            s_y[threadIdx.x] = __float_as_int(yv);
            s_cb[threadIdx.x] = cb;
            s_ct[threadIdx.x] = ct;
            s_pn[threadIdx.x] = cb + ct;
#pragma unroll
            for (int k = 0; k < kMaxDurCols; ++k)
                if (k < a.n_dur) s_gd[threadIdx.x * kMaxDurCols + k] = gd[k];
        }
        __syncthreads();
        const uint32_t items = (uint32_t)R * P.groups;
        // the tile's stash and G rows, addressed with 32-bit offsets from here
        const char* sbase = static_cast<const char*>(P.stash.data) + row0 * g.vpad * kES;
        __nv_bfloat16* gbase = P.G + (int64_t)r0 * g.gw;
        for (uint32_t f0 = threadIdx.x; f0 < items; f0 += kStashThreads * kBatch) {
            uint4 raw[kBatch][kLoads];
#pragma unroll
            for (int k = 0; k < kBatch; ++k) {
                const uint32_t f = f0 + (uint32_t)(k * kStashThreads);
                if (f < items) {
                    const uint32_t r = row_of(f, P), q = f - r * P.groups;
                    const uint4* src = reinterpret_cast<const uint4*>(sbase + (r * g.vpad + q * 16) * kES);
#pragma unroll
                    for (int l = 0; l < kLoads; ++l) raw[k][l] = __ldcs(src + l);
                }
            }
#pragma unroll
            for (int k = 0; k < kBatch; ++k) {
                const uint32_t f = f0 + (uint32_t)(k * kStashThreads);
                if (f >= items) break;
                const uint32_t r = row_of(f, P), q = f - r * P.groups;
                const int c0 = (int)q * 16;
                float x[16];  // the stashed values
#pragma unroll
                for (int l = 0; l < kLoads; ++l) {
                    const uint32_t w[4] = {raw[k][l].x, raw[k][l].y, raw[k][l].z, raw[k][l].w};
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        if (PARTS == 1) {
                            const float2 h2 = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
                            x[8 * l + 2 * i] = h2.x;
                            x[8 * l + 2 * i + 1] = h2.y;
                        } else {
                            x[4 * l + i] = __uint_as_float(w[i]);
                        }
                    }
                }
                const float e = s_e[r * kStashMaxChunks + (P.magic_chunk ? __umulhi(q, P.magic_chunk) : q)];
                const float pn = s_pn[r];
                float gv[16];
                if (c0 + 16 <= a.V) {  // token columns: softmax * (cb + ct), then the two edges
#pragma unroll
                    for (int i = 0; i < 16; ++i) gv[i] = ex2_fast(fmaf(x[i], kLog2e, e)) * pn;
                    const int y = s_y[r];
                    if ((unsigned)(a.blank - c0) < 16u || (unsigned)(y - c0) < 16u) {  // few items
                        const float cb = s_cb[r], ct = s_ct[r];
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            if (c0 + i == a.blank) gv[i] -= cb;
                            if (c0 + i == y) gv[i] -= ct;
                        }
                    }
                } else {  // the row's last columns: tokens, duration-logit gradients, padding
                    const int y = s_y[r];
                    const float cb = s_cb[r], ct = s_ct[r];
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const int cc = c0 + i;
                        float v = 0.f;
                        if (cc < a.V) {
                            v = ex2_fast(fmaf(x[i], kLog2e, e)) * pn;
                            if (cc == a.blank) v -= cb;
                            if (cc == y) v -= ct;
                        } else if (cc < Vf) {
                            v = s_gd[r * kMaxDurCols + (cc - a.V)];
                        }
                        gv[i] = v;
                    }
                }
                __nv_bfloat16* grow = gbase + r * g.gw + c0;
                if (PARTS == 1) {
                    st_global_32B(grow, make_uint4(pack_bf16(gv[0], gv[1]), pack_bf16(gv[2], gv[3]),
                                                   pack_bf16(gv[4], gv[5]), pack_bf16(gv[6], gv[7])),
                                  make_uint4(pack_bf16(gv[8], gv[9]), pack_bf16(gv[10], gv[11]),
                                             pack_bf16(gv[12], gv[13]), pack_bf16(gv[14], gv[15])));
                } else {  // split fp32: [hi | hi | lo]
                    float lo[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const float h = __bfloat162float(__float2bfloat16_rn(gv[i]));
                        lo[i] = gv[i] - h;
                        gv[i] = h;
                    }
                    const uint4 h0 = make_uint4(pack_bf16(gv[0], gv[1]), pack_bf16(gv[2], gv[3]),
                                                pack_bf16(gv[4], gv[5]), pack_bf16(gv[6], gv[7]));
                    const uint4 h1 = make_uint4(pack_bf16(gv[8], gv[9]), pack_bf16(gv[10], gv[11]),
                                                pack_bf16(gv[12], gv[13]), pack_bf16(gv[14], gv[15]));
                    st_global_32B(grow, h0, h1);
                    st_global_32B(grow + g.vpad, h0, h1);
                    st_global_32B(grow + 2 * g.vpad,
                                  make_uint4(pack_bf16(lo[0], lo[1]), pack_bf16(lo[2], lo[3]),
                                             pack_bf16(lo[4], lo[5]), pack_bf16(lo[6], lo[7])),
                                  make_uint4(pack_bf16(lo[8], lo[9]), pack_bf16(lo[10], lo[11]),
                                             pack_bf16(lo[12], lo[13]), pack_bf16(lo[14], lo[15])));
                }
            }
        }
    }
    // zero rows that pad the pass to whole 128-row tiles
    const int zgroups = g.gw / 8;
    for (int64_t i = (int64_t)blockIdx.x * kStashThreads + threadIdx.x; i < (int64_t)zrows * zgroups;
         i += (int64_t)gridDim.x * kStashThreads)
        *reinterpret_cast<uint4*>(P.G + (int64_t)(rows + i / zgroups) * g.gw + (i % zgroups) * 8) = make_uint4(0, 0, 0, 0);
}

}  // namespace

// =================================================================== backward
//
// Per pass of nodes [s, e) (bounds computed on the device): the dlogits kernel
// above writes G = d loss / d logits (bf16 rows of the pass) and H = hidden
// (bf16); then
//   dH  kernel: the transposed product D^T = Wf^T G^T per (128-wide hidden
//               slice, 256-node tile): M = 128 hidden columns on the TMEM
//               lanes, N = 256 consecutive nodes on the TMEM columns, K = the
//               vocabulary. Each epilogue thread owns one hidden column, so both
//               reductions of d_hidden = D ⊙ (1 - h^2) are thread-private:
//               d_enc[b, t] is a running sum over the contiguous label positions
//               of frame t (one global add per frame), d_dec[b, u] accumulates in
//               the thread's own column of a shared-memory row block of the
//               current utterance (flushed with one global add per element
//               when the utterance ends). h = tanh(enc + dec) is recomputed from
//               the fp32 activations (a register copy of the frame's enc value
//               and a shared copy of the utterance's dec rows).
//   dW  kernel: split-K over the pass rows, D = G^T H (M = 128 vocabulary rows,
//               N = 320 hidden columns as 192 + 128, both operands MN-major from G
//               and H), added to dW / dW_dur once per CTA.

namespace {

constexpr int kDhM = 128;                          // hidden columns per work item (UMMA M)
constexpr int kDhNodes = 256;                      // nodes per tile (UMMA N)
constexpr int kDhK = 32;                           // vocabulary per stage (64 B rows)
constexpr int kDhABytes = kDhM * kDhK * 2;         // 8 KB; a stage adds the G rows (16 KB, 8 KB per CTA of a pair):
                                                   // 4 stages of 24 KB beat 2 of 48 KB here
constexpr int kDwM = 128;         // vocabulary rows per dW work item (UMMA M)
constexpr int kDwN = 320;         // hidden columns per dW work item (UMMA N = 192 + 128)
constexpr int kBwdThreads = 192;  // TMA, MMA, 4 epilogue warps
constexpr int kDwStageBytes = (2 + kDwN / 64) * 64 * 64 * 2;  // 2 + 5 boxes of 64 x 64, 56 KB
struct DhParams {
    JointArgs a;
    Geom g;
    const int32_t* bounds;
    int pass;
    int stages;
    int ndt;       // hidden slices of kDhM columns
    int groups;    // node-range groups; CTA i works on slice i % ndt of range i / ndt
    int dec_rows;  // label rows of the shared dec copy / d_dec accumulator (0: global path)
    float* d_enc;
    float* d_dec;
    int* err;
};

// One activation as fp32 from the fp32 or the bf16 copy.
__device__ __forceinline__ float act(const float* f32, const __nv_bfloat16* b16, int64_t i) {
    return b16 ? __bfloat162float(b16[i]) : __ldg(f32 + i);
}

// Walk state of one epilogue thread over consecutive nodes (warp-uniform except
// the per-column values).
__device__ __forceinline__ float dec_value(float x) { return x; }
__device__ __forceinline__ float dec_value(__nv_bfloat16 x) { return __bfloat162float(x); }

struct DhWalk {
    int b, t, u, Tb, Ub;
    float e_cur, e_nxt;  // enc[b, t, col], enc[b, t + 1, col]
    float acc_e;         // running d_enc sum of frame t
    bool dirty;          // d_dec rows of utterance b hold unflushed sums
};

template <bool kSmemDec, bool kSplit>
struct DhEpilogue {
    const DhParams& P;
    const int col;     // hidden column
    const bool col_ok;
    const int cl;      // column within the slice (shared-memory column)
    // [dec_rows][kDhM] dec copy: bf16 on the bf16 path (it only enters tanh(enc + dec),
    // far below the path's rounding), which leaves shared memory for another ring stage
    using DecT = typename std::conditional<kSplit, float, __nv_bfloat16>::type;
    DecT* sdin;
    float* sacc;       // [dec_rows][kDhM] d_dec sums

    // h = tanh(enc + dec), recomputed as the hidden rows computed it
    __device__ __forceinline__ float th(float x) const { return kSplit ? tanhf(x) : tanh_fast(x); }
    __device__ float enc_at(int b, int t) const {
        if (P.a.head) return 0.f;  // CTC head: d hidden itself, no tanh' to recompute
        return col_ok ? act(P.a.enc, P.a.enc16, ((int64_t)b * P.a.T + t) * P.a.d + col) : 0.f;
    }
    __device__ float dec_at(const DhWalk& w, int u) const {
        if (kSmemDec) return dec_value(sdin[u * kDhM + cl]);
        return col_ok ? act(P.a.dec, P.a.dec16, ((int64_t)w.b * P.a.U + u) * P.a.d + col) : 0.f;
    }
    __device__ void add_dec(const DhWalk& w, int u, float x) const {
        if (kSmemDec)
            sacc[u * kDhM + cl] += x;
        else if (col_ok)
            atomicAdd(P.d_dec + ((int64_t)w.b * P.a.U + u) * P.a.d + col, x);
    }
    // Enter utterance b at frame t (label position 0 follows from the caller).
    __device__ void enter(DhWalk& w, int b, int t) const {
        w.b = b;
        w.t = t;
        w.Tb = __ldg(P.a.m.Tb + b);
        w.Ub = __ldg(P.a.m.Ub + b);
        w.e_cur = enc_at(b, t);
        w.e_nxt = t + 1 < w.Tb ? enc_at(b, t + 1) : 0.f;
        if (kSmemDec) {
            // 16 label positions' loads in flight before their shared-memory stores
            // (a load behind each store would pay one memory latency per position)
            for (int u0 = 0; u0 < w.Ub; u0 += 16) {
                float v[16];
#pragma unroll
                for (int i = 0; i < 16; ++i)
                    v[i] = (col_ok && u0 + i < w.Ub)
                               ? act(P.a.dec, P.a.dec16, ((int64_t)b * P.a.U + u0 + i) * P.a.d + col)
                               : 0.f;
#pragma unroll
                for (int i = 0; i < 16; ++i)
                    if (u0 + i < w.Ub) {
                        sdin[(u0 + i) * kDhM + cl] = DecT(v[i]);
                        sacc[(u0 + i) * kDhM + cl] = 0.f;
                    }
            }
        }
        w.dirty = false;
    }
    __device__ void flush_dec(DhWalk& w) const {
        if (kSmemDec && w.dirty && col_ok)
            for (int u = 0; u < w.Ub; ++u)
                atomicAdd(P.d_dec + ((int64_t)w.b * P.a.U + u) * P.a.d + col, sacc[u * kDhM + cl]);
        w.dirty = false;
    }
    __device__ void flush_enc(DhWalk& w) const {
        if (col_ok) atomicAdd(P.d_enc + ((int64_t)w.b * P.a.T + w.t) * P.a.d + col, w.acc_e);
        w.acc_e = 0.f;
    }
    // Frame t of the walk is complete: move to the next frame (or utterance).
    __device__ void end_frame(DhWalk& w) const {
        flush_enc(w);
        w.u = 0;
        if (++w.t < w.Tb) {
            w.e_cur = w.e_nxt;
            w.e_nxt = w.t + 1 < w.Tb ? enc_at(w.b, w.t + 1) : 0.f;
            return;
        }
        flush_dec(w);
        int b = w.b + 1;
        while (b < P.a.B && __ldg(P.a.m.Tb + b) == 0) ++b;
        if (b < P.a.B) enter(w, b, 0);
        else w.b = P.a.B;  // past the last node
    }
    // One node at a time (any U_b, utterance changes inside the group).
    __device__ void node(DhWalk& w, float g) const {
        if (P.a.head) {  // CTC head: one node per frame, d_hidden = G Wf
            w.acc_e += g;
            if (++w.u == w.Ub) end_frame(w);
            return;
        }
        const float h = th(w.e_cur + dec_at(w, w.u));
        const float x = g * (1.f - h * h);
        w.acc_e += x;
        add_dec(w, w.u, x);
        w.dirty = true;
        if (++w.u == w.Ub) end_frame(w);
    }
    // N consecutive nodes (N = 16 or 32) with U_b >= N that stay inside utterance
    // b: the N label positions are distinct, so their d_dec rows load and store
    // together, and at most one frame boundary falls inside the group. The N
    // node chains are independent, so a larger N gives the single epilogue warp
    // of a lane quarter more work to overlap its latencies with; the frame sums
    // are pairwise trees.
    template <int N>
    __device__ void group(DhWalk& w, const float (&v)[N]) const {
        const int k = w.Ub - w.u;  // nodes left in frame t (at most one frame boundary here)
        if (k >= N) {
            // the whole group inside frame t (most groups): label positions u .. u + N - 1,
            // one base address with constant offsets, no per-node frame selects
            const DecT* din = sdin + w.u * kDhM + cl;
            float* acc = sacc + w.u * kDhM + cl;
            float dv[N], sa[N], xs[N];
#pragma unroll
            for (int i = 0; i < N; ++i) dv[i] = dec_value(din[i * kDhM]);
#pragma unroll
            for (int i = 0; i < N; ++i) sa[i] = acc[i * kDhM];
#pragma unroll
            for (int i = 0; i < N; ++i) {
                const float h = th(w.e_cur + dv[i]);
                xs[i] = v[i] * (1.f - h * h);
                acc[i * kDhM] = sa[i] + xs[i];
            }
#pragma unroll
            for (int s2 = 1; s2 < N; s2 *= 2)
#pragma unroll
                for (int i = 0; i + s2 < N; i += 2 * s2) xs[i] += xs[i + s2];
            w.acc_e += xs[0];
            w.dirty = true;
            w.u += N;
            if (w.u == w.Ub) end_frame(w);
            return;
        }
        int idx[N];
#pragma unroll
        for (int i = 0; i < N; ++i) {
            int ui = w.u + i;
            if (ui >= w.Ub) ui -= w.Ub;
            idx[i] = ui * kDhM + cl;
        }
        float dv[N], sa[N];
#pragma unroll
        for (int i = 0; i < N; ++i) dv[i] = dec_value(sdin[idx[i]]);
#pragma unroll
        for (int i = 0; i < N; ++i) sa[i] = sacc[idx[i]];
        float lo[N], hi[N];
#pragma unroll
        for (int i = 0; i < N; ++i) {
            const float h = th((i < k ? w.e_cur : w.e_nxt) + dv[i]);
            const float x = v[i] * (1.f - h * h);
            sacc[idx[i]] = sa[i] + x;
            lo[i] = i < k ? x : 0.f;
            hi[i] = i < k ? 0.f : x;
        }
#pragma unroll
        for (int s2 = 1; s2 < N; s2 *= 2)
#pragma unroll
            for (int i = 0; i + s2 < N; i += 2 * s2) {
                lo[i] += lo[i + s2];
                hi[i] += hi[i + s2];
            }
        w.dirty = true;
        if (k < N) {  // frame t ends inside the group; frame t + 1 is in the same utterance
            w.acc_e += lo[0];
            flush_enc(w);
            ++w.t;
            w.e_cur = w.e_nxt;
            w.e_nxt = w.t + 1 < w.Tb ? enc_at(w.b, w.t + 1) : 0.f;
            w.acc_e = hi[0];
            w.u = N - k;
        } else {
            w.acc_e += lo[0];
            w.u += N;
            if (w.u == w.Ub) end_frame(w);
        }
    }
};

// kCta = 2: a CTA pair (cluster of two, cta_group::2) runs one M = 256 MMA over
// two hidden slices: each CTA streams its own slice of the transposed weight
// (A) and half of the node tile's G rows (B), and keeps its slice's 128 x 256
// accumulator in its own TMEM, so the epilogue is the single-CTA one. Per SM a
// stage carries a third fewer bytes for the same MMA time. With an odd slice
// count the last pair's second CTA has no slice: its weight rows are past the
// hidden width (the loads fill zeros) and its epilogue only releases buffers.
template <bool kSmemDec, bool kSplit, int kCta = 1>
__global__ void __launch_bounds__(kBwdThreads, 1)
    tc_dh_kernel(const __grid_constant__ CUtensorMap map_wt, const __grid_constant__ CUtensorMap map_g, DhParams P) {
    constexpr int SB = kDhABytes + (kDhNodes / kCta) * kDhK * 2;  // stage: A slice + this CTA's G rows
    extern __shared__ uint8_t smem_raw[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const JointArgs& a = P.a;
    const int S = P.stages;
    uint8_t* stages = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    using DecT = typename DhEpilogue<kSmemDec, kSplit>::DecT;
    DecT* sdin = reinterpret_cast<DecT*>(stages + (size_t)S * SB);  // [dec_rows][kDhM]
    float* sacc = reinterpret_cast<float*>(sdin + (size_t)P.dec_rows * kDhM);  // [dec_rows][kDhM]
    uint64_t* bars = reinterpret_cast<uint64_t*>(sacc + (size_t)P.dec_rows * kDhM);  // 512 B multiples: aligned
    uint64_t* b_full = bars;
    uint64_t* b_empty = bars + S;
    uint64_t* t_full = bars + 2 * S;
    uint64_t* t_empty = t_full + 2;
    uint64_t* done = t_empty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    int* err = P.err;

    const int s = P.bounds[P.pass], e = P.bounds[P.pass + 1];
    const uint32_t rank = kCta == 2 ? cluster_ctarank() : 0;
    const bool leader = rank == 0;
    // work item: hidden slice dt of node-range group grp (a pair: slices 2 j and 2 j + 1)
    const int nslot = kCta == 2 ? (P.ndt + 1) / 2 : P.ndt;
    const int unit = (int)blockIdx.x / kCta;
    const int dt = kCta == 2 ? 2 * (unit % nslot) + (int)rank : unit % nslot;
    const int grp = unit / nslot;
    const bool slice_ok = dt < P.ndt;
    auto in_leader = [&](uint64_t* bar) { return kCta == 2 ? mapa_shared(smem_u32(bar), 0) : smem_u32(bar); };
    auto in_peer = [&](uint64_t* bar) { return mapa_shared(smem_u32(bar), 1); };
    const int ntiles = e > s ? (e - s + kDhNodes - 1) / kDhNodes : 0;
    const int tile0 = (int)((int64_t)grp * ntiles / P.groups);
    const int tile1 = (int)((int64_t)(grp + 1) * ntiles / P.groups);
    const int ksteps = (P.g.gw + kDhK - 1) / kDhK;  // K: the vocabulary, over every part

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(&b_full[i], 1);
            mbar_init(&b_empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&t_full[i], 1);
            mbar_init(&t_empty[i], 4 * kCta);  // every epilogue warp of the pair releases the buffer
        }
        mbar_init(done, 1);
        fence_barrier_init();
        prefetch_tensormap(&map_wt);
        prefetch_tensormap(&map_g);
    }
    if (kCta == 2) {
        cluster_sync();  // both CTAs' barriers exist before any cross-CTA arrival
        if (warp == 1) tmem_alloc_pair(tmem_slot, 2 * kDhNodes);
    } else if (warp == 1) {
        tmem_alloc(tmem_slot, 2 * kDhNodes);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            bool issued[8] = {};
            uint32_t ipar[8] = {};
            bool ok = true;
            for (int tile = tile0; ok && tile < tile1; ++tile) {
                for (int k = 0; k < ksteps; ++k) {
                    if (!mbar_wait_cluster(&b_empty[stage], phase ^ 1, err, 11)) {
                        ok = false;
                        break;
                    }
                    uint8_t* st = stages + (size_t)stage * SB;
                    if (kCta == 2) {  // both CTAs' bytes land on the even CTA's barrier
                        if (leader) mbar_arrive_expect_tx(&b_full[stage], 2 * SB);
                        tma_load_2d_pair(st, &map_wt, k * kDhK, dt * kDhM, in_leader(&b_full[stage]));
                        tma_load_2d_pair(st + kDhABytes, &map_g, k * kDhK, tile * kDhNodes + (int)rank * (kDhNodes / 2),
                                         in_leader(&b_full[stage]));
                    } else {
                        mbar_arrive_expect_tx(&b_full[stage], SB);
                        tma_load_2d(st, &map_wt, k * kDhK, dt * kDhM, &b_full[stage]);
                        tma_load_2d(st + kDhABytes, &map_g, k * kDhK, tile * kDhNodes, &b_full[stage]);
                    }
                    issued[stage] = true;
                    ipar[stage] = phase;
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            if (leader)  // the even CTA's full barriers count both CTAs' copies
                for (int i = 0; i < S; ++i)
                    if (issued[i]) mbar_wait_cluster(&b_full[i], ipar[i], err, 12);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------- MMA issuer
        auto commit_both = [&](uint64_t* bar) {
            if (kCta == 2) {
                mma_commit_pair(smem_u32(bar));
                mma_commit_pair(in_peer(bar));
            } else {
                mma_commit(bar);
            }
        };
        if (lane == 0 && leader) {
            const uint32_t idesc = idesc_bf16(kDhM * kCta, kDhNodes, false, false);
            const uint32_t sbase = smem_u32(stages);
            int stage = 0;
            uint32_t phase = 0, q = 0;
            bool ok = true;
            for (int tile = tile0; ok && tile < tile1; ++tile, ++q) {
                const uint32_t buf = q & 1;
                if (!mbar_wait_cluster(&t_empty[buf], ((q >> 1) & 1) ^ 1, err, 13)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                for (int k = 0; k < ksteps; ++k) {
                    if (!mbar_wait_cluster(&b_full[stage], phase, err, 14)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t st = sbase + stage * SB;
#pragma unroll
                    for (int kk = 0; kk < kDhK / 16; ++kk) {
                        const uint64_t ad = desc_k64(st + kk * 32), bd = desc_k64(st + kDhABytes + kk * 32);
                        if (kCta == 2)
                            mma_bf16_pair(tmem_base + buf * kDhNodes, ad, bd, idesc, (k | kk) != 0 ? 1u : 0u);
                        else
                            mma_bf16(tmem_base + buf * kDhNodes, ad, bd, idesc, (k | kk) != 0 ? 1u : 0u);
                    }
                    commit_both(&b_empty[stage]);
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (ok) commit_both(&t_full[buf]);
            }
            commit_both(done);
            mbar_wait(done, 0, err, 15);
        } else if (kCta == 2 && lane == 0) {
            mbar_wait_cluster(done, 0, err, 15);  // odd CTA: the even CTA's MMAs write this TMEM
        }
    } else if (tile1 > tile0 && !slice_ok) {
        // a pair's CTA without a hidden slice: release each accumulator buffer
        uint32_t q = 0;
        for (int tile = tile0; tile < tile1; ++tile, ++q) {
            const uint32_t buf = q & 1;
            if (!__all_sync(0xffffffffu, mbar_wait_cluster(&t_full[buf], (q >> 1) & 1, err, 16))) break;
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(in_leader(&t_empty[buf]));
        }
    } else if (tile1 > tile0) {
        // ------------------------------------------------------------------- epilogue
        const int lane_base = 32 * (warp & 3);
        const int cl = lane_base + lane;
        const int col = dt * kDhM + cl;
        const DhEpilogue<kSmemDec, kSplit> ep{P, col, col < a.d, cl, sdin, sacc};
        DhWalk w;
        {
            const int n0 = s + tile0 * kDhNodes;
            const NodeCoord c = node_coord(a.m, a.B, n0);
            w.acc_e = 0.f;
            ep.enter(w, c.b, c.t);
            w.u = c.u;
        }
        uint32_t q = 0;
        bool ok = true;
        for (int tile = tile0; tile < tile1; ++tile, ++q) {
            const uint32_t buf = q & 1;
            if (!__all_sync(0xffffffffu, mbar_wait_cluster(&t_full[buf], (q >> 1) & 1, err, 16))) {
                ok = false;
                break;
            }
            tc_fence_after();
            const int cnt = min(kDhNodes, e - (s + tile * kDhNodes));
            const uint32_t taddr = tmem_base + ((uint32_t)lane_base << 16) + buf * kDhNodes;
            for (int g16 = 0; g16 * 16 < cnt;) {
                const int left = cnt - g16 * 16;
                if (kSmemDec && left >= 32 && w.Ub >= 32 && (w.t < w.Tb - 1 || w.Ub - w.u >= 32)) {
                    float v[32];
                    tmem_ld32(taddr + g16 * 16, v);
                    ep.template group<32>(w, v);
                    g16 += 2;
                    continue;
                }
                float v[16];
                tmem_ld16(taddr + g16 * 16, v);
                const bool fast = kSmemDec && left >= 16 && w.Ub >= 16 &&
                                  (w.t < w.Tb - 1 || w.Ub - w.u >= 16);
                if (fast) {
                    ep.template group<16>(w, v);
                } else {
#pragma unroll
                    for (int i = 0; i < 16; ++i)
                        if (i < left) ep.node(w, v[i]);
                }
                ++g16;
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if (kCta == 2)
                    mbar_arrive_cluster(in_leader(&t_empty[buf]));
                else
                    mbar_arrive(&t_empty[buf]);
            }
        }
        // the range may end inside a frame / an utterance: add the partial sums
        if (ok && w.b < a.B) {
            if (w.u > 0) ep.flush_enc(w);
            ep.flush_dec(w);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (kCta == 2) {
        cluster_sync();  // no CTA leaves while its pair may still read its smem or signal it
        tc_fence_after();
        if (warp == 1) tmem_dealloc_pair(tmem_base, 2 * kDhNodes);
    } else {
        tc_fence_after();
        if (warp == 1) tmem_dealloc(tmem_base, 2 * kDhNodes);
    }
}

struct DwParams {
    JointArgs a;
    Geom g;
    const int32_t* bounds;
    int pass;
    int splits;
    float* dW;
    float* dWd;
    float* dbias;  // CTC head: column d of the product (the ones column)
    int* err;
};

constexpr int kDwStages = 4;

__global__ void __launch_bounds__(kBwdThreads, 1)
    tc_dw_kernel(const __grid_constant__ CUtensorMap map_g, const __grid_constant__ CUtensorMap map_h, DwParams P) {
    extern __shared__ uint8_t smem_raw[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t* stages = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(stages + (size_t)kDwStages * kDwStageBytes);
    uint64_t* b_full = bars;
    uint64_t* b_empty = bars + kDwStages;
    uint64_t* t_full = bars + 2 * kDwStages;
    uint64_t* done = t_full + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    int* err = P.err;

    const int nvt = (P.g.vpad + kDwM - 1) / kDwM;
    const int nkt = (P.g.kp + kDwN - 1) / kDwN;
    const int item = blockIdx.x;
    // split slowest: the CTAs of one row range run side by side and share its G / H rows in L2
    const int vt = item % nvt;
    const int kt = (item / nvt) % nkt;
    const int split = item / (nvt * nkt);
    const int s = P.bounds[P.pass], e = P.bounds[P.pass + 1];
    const int rows = e > s ? (e - s + 63) / 64 * 64 : 0;  // zero rows pad the pass to 64
    const int per = ((rows / 64 + P.splits - 1) / P.splits) * 64;
    const int r0 = split * per, r1 = min(rows, r0 + per);
    // split fp32: one pass over the rows per part p, G block p against H block p
    const int rsteps = (vt < nvt && r1 > r0) ? (r1 - r0) / 64 : 0;
    const int nsteps = rsteps * P.g.parts;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kDwStages; ++i) {
            mbar_init(&b_full[i], 1);
            mbar_init(&b_empty[i], 1);
        }
        mbar_init(t_full, 1);
        mbar_init(done, 1);
        fence_barrier_init();
        prefetch_tensormap(&map_g);
        prefetch_tensormap(&map_h);
    }
    if (warp == 1) tmem_alloc(tmem_slot, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    constexpr int kBox = 64 * 64 * 2;  // one 64 x 64 bf16 TMA box

    if (warp == 0) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            bool issued[kDwStages] = {};
            uint32_t ipar[kDwStages] = {};
            for (int i = 0; i < nsteps; ++i) {
                if (!mbar_wait(&b_empty[stage], phase ^ 1, err, 21)) break;
                uint8_t* st = stages + (size_t)stage * kDwStageBytes;
                const int part = i / rsteps;
                const int r = r0 + (i - part * rsteps) * 64;
                const int gc = part * P.g.vpad + vt * kDwM;  // G columns of this part
                mbar_arrive_expect_tx(&b_full[stage], kDwStageBytes);
                tma_load_2d(st, &map_g, gc, r, &b_full[stage]);
                tma_load_2d(st + kBox, &map_g, gc + 64, r, &b_full[stage]);
                // H: kDwN / 64 column blocks of 64 in one box of the 3-D view
                tma_load_3d(st + 2 * kBox, &map_h, 0, r, part * (P.g.kp / 64) + kt * (kDwN / 64), &b_full[stage]);
                issued[stage] = true;
                ipar[stage] = phase;
                if (++stage == kDwStages) {
                    stage = 0;
                    phase ^= 1;
                }
            }
            for (int i = 0; i < kDwStages; ++i)
                if (issued[i]) mbar_wait(&b_full[i], ipar[i], err, 22);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // N = 320 as 192 + 128 (both start on a 64-column block; an N = 64 MMA
            // would be issue-bound)
            const uint32_t id_a = idesc_bf16(kDwM, 192, true, true);
            const uint32_t id_b = idesc_bf16(kDwM, 128, true, true);
            const uint32_t sbase = smem_u32(stages);
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int i = 0; i < nsteps; ++i) {
                if (!mbar_wait(&b_full[stage], phase, err, 23)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t st = sbase + stage * kDwStageBytes;
#pragma unroll
                for (int ks = 0; ks < 4; ++ks) {  // 16 rows (K) per MMA
                    const uint64_t ad = desc_mn128(st + ks * 2048, kBox);
                    const uint64_t b0 = desc_mn128(st + 2 * kBox + ks * 2048, kBox);
                    const uint64_t b1 = desc_mn128(st + 5 * kBox + ks * 2048, kBox);
                    const uint32_t acc = (i | ks) != 0 ? 1u : 0u;
                    mma_bf16(tmem_base, ad, b0, id_a, acc);
                    mma_bf16(tmem_base + 192, ad, b1, id_b, acc);
                }
                mma_commit(&b_empty[stage]);
                if (++stage == kDwStages) {
                    stage = 0;
                    phase ^= 1;
                }
            }
            if (ok) mma_commit(t_full);
            mma_commit(done);
            mbar_wait(done, 0, err, 24);
        }
    } else if (nsteps > 0) {
        // --------------------------------------------------------------- epilogue
        const int lane_base = 32 * (warp & 3);
        const int v = vt * kDwM + lane_base + lane;
        const JointArgs& a = P.a;
        const bool ok = __all_sync(0xffffffffu, mbar_wait(t_full, 0, err, 25));
        tc_fence_after();
        if (ok) {
            float* dst = nullptr;
            if (v < a.V)
                dst = P.dW + (int64_t)v * a.d;
            else if (v < a.V + a.n_dur)
                dst = P.dWd + (int64_t)(v - a.V) * a.d;
            const uint32_t taddr = tmem_base + ((uint32_t)lane_base << 16);
            for (int gi = 0; gi < kDwN / 16; ++gi) {
                float acc[16];
                tmem_ld16(taddr + gi * 16, acc);
                if (dst) {
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const int k = kt * kDwN + gi * 16 + i;
                        if (k < a.d)
                            atomicAdd(dst + k, acc[i]);
                        else if (k == a.d && P.dbias && v < a.V)
                            atomicAdd(P.dbias + v, acc[i]);
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem_base, 512);
}

// ---------------------------------------------------------- backward host side

struct BwdLayout {
    int64_t step;  // nodes per pass (multiple of kPassAlign = kDhNodes) = rows of the G / H buffers
    int passes;
    size_t wf, wt, g, h, bounds, err, total;
};

BwdLayout bwd_layout(const JointArgs& a, int64_t cap) {
    const Geom g = make_geom(a);
    BwdLayout L;
    const PassPlan pp = pass_plan(cap);
    L.step = pp.step;
    L.passes = pp.passes;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t o = off;
        off += al256(bytes);
        return o;
    };
    L.wf = take(sizeof(__nv_bfloat16) * (size_t)g.vpad * g.kpad);
    L.wt = take(sizeof(__nv_bfloat16) * (size_t)g.kp * g.gw);
    L.g = take(sizeof(__nv_bfloat16) * (size_t)L.step * g.gw);
    L.h = take(sizeof(__nv_bfloat16) * (size_t)L.step * g.kpad);
    L.bounds = take(sizeof(int32_t) * (L.passes + 1));
    L.err = take(sizeof(int));
    L.total = off;
    return L;
}

size_t dh_smem_bytes(int stages, int dec_rows, int cta = 1, int dec_bytes = 4) {
    const size_t sb = kDhABytes + (size_t)(kDhNodes / cta) * kDhK * 2;
    return 1024 + (size_t)stages * sb + (size_t)(dec_bytes + 4) * dec_rows * kDhM + 8 * (2 * stages + 5) + 16;
}

// CTA pairs for the d_hidden kernel when ASR_B200_DH_PAIRS=1. Off by default:
// on B200 the pairs measured slower at config 5 (26.9 vs 22.5 ms, one CTA in
// six without a slice at d = 640) and at config 4 (9.6 vs 8.9 ms, none idle).
bool dh_pairs() {
    static const bool pairs = [] {
        const char* e = std::getenv("ASR_B200_DH_PAIRS");
        return e && e[0] == '1';
    }();
    return pairs;
}

size_t dw_smem_bytes() { return 1024 + (size_t)kDwStages * kDwStageBytes + 8 * (2 * kDwStages + 2) + 16; }

}  // namespace

bool tc_backward_supported(const JointArgs& a) {
    if (!tc_supported(a)) return false;
    return (int)dh_smem_bytes(2, 0) <= dyn_smem_limit() && (int)dw_smem_bytes() <= dyn_smem_limit();
}

size_t tc_backward_scratch_bytes(const JointArgs& a, int node_capacity) {
    return bwd_layout(a, node_capacity).total + 256;
}

int tc_joint_backward(const JointArgs& a, const JointBwdIn& in, const JointBwdOut& o, int node_capacity, void* scratch,
                      size_t scratch_bytes, cudaStream_t st, const LogitStash& stash) {
    const Geom g = make_geom(a);
    const BwdLayout L = bwd_layout(a, node_capacity);
    if (scratch_bytes < L.total) return ASR_ERR_WORKSPACE;
    char* base = reinterpret_cast<char*>(scratch);
    auto* Wf = reinterpret_cast<__nv_bfloat16*>(base + L.wf);
    auto* Wt = reinterpret_cast<__nv_bfloat16*>(base + L.wt);
    auto* G = reinterpret_cast<__nv_bfloat16*>(base + L.g);
    auto* H = reinterpret_cast<__nv_bfloat16*>(base + L.h);
    auto* bounds = reinterpret_cast<int32_t*>(base + L.bounds);
    int* err = reinterpret_cast<int*>(base + L.err);
    const int sms = sm_count();
    ASR_CUDA_TRY(cudaMemsetAsync(err, 0, sizeof(int), st));
    {
        KernelTimer kt("joint_prep_weights", st);
        prep_weights_kernel<<<sms * 4, 256, 0, st>>>(a.W, a.Wd, a.head ? a.bias : nullptr, a.V, a.n_dur, a.d,
                                                     g.vpad, g.kp, g.parts, Wf, Wt);
        ASR_LAUNCH_CHECK();
    }
    {
        KernelTimer kt("joint_plan_passes", st);
        plan_passes_kernel<<<(L.passes + 1 + 127) / 128, 128, 0, st>>>(a.m, a.B, L.passes, L.step, bounds);
        ASR_LAUNCH_CHECK();
    }
    // tensor maps
    const int rows = (int)L.step;
    const bool pairs = joint_pairs() && !joint_stream(g);  // pairs use the resident hidden tile
    CUtensorMap mfull, mtail, m_h, m_wt, m_g, m_gmn, m_hmn;
    if (!joint_weight_maps(g, Wf, pairs, &mfull, &mtail)) return ASR_ERR_CUDA;
    if (!make_map(&m_h, H, rows, g.kpad, kAK, kBM, CU_TENSOR_MAP_SWIZZLE_128B)) return ASR_ERR_CUDA;
    if (!make_map(&m_wt, Wt, g.kp, g.gw, kDhK, kDhM, CU_TENSOR_MAP_SWIZZLE_64B)) return ASR_ERR_CUDA;
    if (!make_map(&m_g, G, rows, g.gw, kDhK, kDhNodes, CU_TENSOR_MAP_SWIZZLE_64B)) return ASR_ERR_CUDA;
    if (!make_map(&m_gmn, G, rows, g.gw, 64, 64, CU_TENSOR_MAP_SWIZZLE_128B)) return ASR_ERR_CUDA;
    if (!make_map_blocks(&m_hmn, H, rows, g.kpad, 64, kDwN / 64)) return ASR_ERR_CUDA;

    // dlogits kernel parameters
    TcParams TP;
    std::memset(&TP, 0, sizeof(TP));
    TP.a = a;
    TP.g = g;
    TP.bwd = in;
    TP.G = G;
    TP.range.bounds = bounds;
    TP.err = err;
    const size_t smem_fw = smem_bytes_for(g.kchunks);
    const bool use_stash = stash.nodes > 0 && !a.head;
    if (use_stash) TP.stash = stash;
    StashParams SP;
    std::memset(&SP, 0, sizeof(SP));
    SP.a = a;
    SP.g = g;
    SP.bounds = bounds;
    SP.stash = TP.stash;
    SP.in = in;
    SP.G = G;
    SP.groups = (uint32_t)(g.vpad / 16);
    // ceil(2^32 / D), exact for every item index below 2^32 / D; 0 stands for D = 1
    auto magic = [](uint32_t D) { return D == 1 ? 0u : (uint32_t)(((1ull << 32) + D - 1) / D); };
    SP.magic_row = magic(SP.groups);
    SP.magic_chunk = magic((uint32_t)(g.cw / 16));
    // every node below the capacity stashed: the recompute kernel has no work
    const bool recompute = !use_stash || (int64_t)stash.nodes < (int64_t)node_capacity;

    // dH parameters: shared dec rows for the whole label range when they fit,
    // then the deepest pipeline that still fits
    DhParams DP;
    std::memset(&DP, 0, sizeof(DP));
    DP.a = a;
    DP.g = g;
    DP.bounds = bounds;
    DP.d_enc = o.d_enc;
    DP.d_dec = o.d_dec;
    DP.err = err;
    DP.ndt = (g.kp + kDhM - 1) / kDhM;
    // CTA pairs take two hidden slices per node tile (the CTC head keeps single CTAs)
    const int dh_cta = dh_pairs() && !a.head && DP.ndt > 1 ? 2 : 1;
    const int dh_units = dh_cta == 2 ? (DP.ndt + 1) / 2 : DP.ndt;  // work items per node range
    DP.groups = std::max(1, sms / (dh_units * dh_cta));
    const int limit = dyn_smem_limit();
    const int dec_bytes = g.parts == 3 ? 4 : 2;  // the shared dec copy: fp32 on the split path, bf16 otherwise
    DP.dec_rows = !a.head && (int)dh_smem_bytes(2, a.U, dh_cta, dec_bytes) <= limit ? a.U : 0;
    DP.stages = 2;
    while (DP.stages < 8 && (int)dh_smem_bytes(DP.stages + 1, DP.dec_rows, dh_cta, dec_bytes) <= limit) ++DP.stages;
    const size_t smem_dh = dh_smem_bytes(DP.stages, DP.dec_rows, dh_cta, dec_bytes);
    auto dh_kernel = dh_cta == 2
                         ? (g.parts == 3 ? (DP.dec_rows > 0 ? tc_dh_kernel<true, true, 2> : tc_dh_kernel<false, true, 2>)
                                         : (DP.dec_rows > 0 ? tc_dh_kernel<true, false, 2> : tc_dh_kernel<false, false, 2>))
                         : (g.parts == 3 ? (DP.dec_rows > 0 ? tc_dh_kernel<true, true> : tc_dh_kernel<false, true>)
                                         : (DP.dec_rows > 0 ? tc_dh_kernel<true, false> : tc_dh_kernel<false, false>));
    ASR_CUDA_TRY(cudaFuncSetAttribute(dh_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_dh));
    CUtensorMap m_g2;  // the pair's half tiles of G rows
    if (dh_cta == 2 && !make_map(&m_g2, G, rows, g.gw, kDhK, kDhNodes / 2, CU_TENSOR_MAP_SWIZZLE_64B))
        return ASR_ERR_CUDA;

    DwParams WP;
    std::memset(&WP, 0, sizeof(WP));
    WP.a = a;
    WP.g = g;
    WP.bounds = bounds;
    WP.dW = o.dW;
    WP.dWd = o.dWd;
    WP.dbias = a.head ? o.dbias : nullptr;
    WP.err = err;
    const int nvt = (g.vpad + kDwM - 1) / kDwM, nkt = (g.kp + kDwN - 1) / kDwN;
    WP.splits = std::max(1, sms / (nvt * nkt));  // one wave: a CTA fills an SM's shared memory
    const size_t smem_dw = dw_smem_bytes();
    ASR_CUDA_TRY(cudaFuncSetAttribute(tc_dw_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_dw));

    for (int p = 0; p < L.passes; ++p) {
        TP.range.pass = p;
        SP.pass = p;
        DP.pass = p;
        WP.pass = p;
        {
            int rc = launch_hidden(a, g, bounds, p, H, st);
            if (rc != ASR_OK) return rc;
        }
        if (use_stash) {
            KernelTimer kt("joint_dlogits_stash", st);
            // one resident wave: the CTAs stride over the pass's tiles
            auto kern = g.parts == 1 ? stash_dlogits_kernel<1> : stash_dlogits_kernel<3>;
            int per_sm = 1;
            ASR_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kStashThreads, 0));
            kern<<<sms * std::max(per_sm, 1), kStashThreads, 0, st>>>(SP);
            ASR_LAUNCH_CHECK();
        }
        if (recompute) {
            KernelTimer kt("joint_dlogits_tc", st);
            int rc = launch_joint<true>(pairs, L.step / kBM, smem_fw, mfull, mtail, m_h, TP, st);
            if (rc != ASR_OK) return rc;
        }
        {
            KernelTimer kt("joint_dhidden_tc", st);
            if (dh_cta == 2) {
                cudaLaunchConfig_t cfg = {};
                cfg.gridDim = dim3(DP.groups * dh_units * 2);
                cfg.blockDim = dim3(kBwdThreads);
                cfg.dynamicSmemBytes = smem_dh;
                cfg.stream = st;
                cudaLaunchAttribute attr[1];
                attr[0].id = cudaLaunchAttributeClusterDimension;
                attr[0].val.clusterDim.x = 2;
                attr[0].val.clusterDim.y = 1;
                attr[0].val.clusterDim.z = 1;
                cfg.attrs = attr;
                cfg.numAttrs = 1;
                ASR_CUDA_TRY(cudaLaunchKernelEx(&cfg, dh_kernel, m_wt, m_g2, DP));
            } else {
                dh_kernel<<<DP.groups * DP.ndt, kBwdThreads, smem_dh, st>>>(m_wt, m_g, DP);
                ASR_LAUNCH_CHECK();
            }
        }
        {
            KernelTimer kt("joint_dweight_tc", st);
            tc_dw_kernel<<<nvt * nkt * WP.splits, kBwdThreads, smem_dw, st>>>(m_gmn, m_hmn, WP);
            ASR_LAUNCH_CHECK();
        }
    }
    return ASR_OK;
}

}  // namespace asr
