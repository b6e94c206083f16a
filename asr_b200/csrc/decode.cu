// Batched greedy transducer decoding (RNN-T and TDT) on sm_100a: the fused
// joint + argmax scan that replaces the reference decoders' per-symbol Python
// joint calls (src/asr/decode/rnnt.py:12-37, src/asr/decode/tdt.py:14-62).
//
// The reference walks one utterance at a time and evaluates
//   token = argmax_v  W[v] . tanh(enc[b, t] + pred)          (system/rnnt.py:29-34)
//   dur   = argmax_c  W_dur[c] . tanh(enc[b, t] + pred)      (system/tdt.py:38-43)
// once per decoding step, re-running the predictor after every emitted token.
// Between two emissions the predictor output of an utterance is fixed, so every
// step until the next emission depends only on the frames it visits. One launch
// of greedy_scan_kernel therefore advances every utterance of the active list
// from its current state to its next emitted token or to its end:
//   * the hidden rows tanh(enc[b, t..t+NF) + pred) of a window of NF frames are
//     built in shared memory (the joint row is never written to HBM);
//   * the window's logits come from one pass over the transposed joint weight
//     (L2-resident, read once per window and reused for all NF frames from
//     registers), each thread owning CPT vocab columns x NF frames;
//   * one utterance is served by a thread-block cluster of C CTAs, CTA r owning
//     the r-th slice of the vocabulary: every CTA reduces its slice to the first
//     maximal index per frame (torch.argmax semantics; NaN counts as the maximum)
//     and stores the candidate into every CTA of the cluster (distributed shared
//     memory, double-buffered by window parity so one cluster barrier per window
//     suffices); every CTA then reduces the C candidates identically. C is
//     chosen per launch from the number of active utterances: C = 1 while they
//     fill the GPU (throughput), up to 4 when few remain (the per-window latency
//     falls with the number of SMs that share the vocabulary);
//   * every CTA replays the reference's state machine over the window (blank
//     advances a frame, TDT durations jump frames, max_symbols_per_frame forces
//     progress), recording every TDT duration, until a token is emitted (the
//     host must run the predictor) or the utterance ends. Frames past the
//     stopping point were computed speculatively and are discarded. Rank 0
//     writes the outputs;
//   * an utterance may scan at most max_windows windows per launch: a long run
//     of blanks pauses and continues in the next launch with the same predictor
//     output, so one utterance's long run does not hold every other utterance's
//     next predictor step.
// The host loop (asr_b200/decode) thus runs one launch per emitted-token level
// instead of one joint call per step and utterance.
#include <algorithm>
#include <climits>
#include <cstdlib>

#include "common.cuh"
#include "tc_common.cuh"

namespace asr {
namespace {

constexpr int kScanThreads = 256;  // 8 warps: two CTAs per SM, four warps per scheduler
constexpr int kScanWarps = kScanThreads / 32;
constexpr int kMaxScanDim = 2048;  // joint dim limit (shared memory: hidden rows + weight ring)
constexpr int kMaxScanDur = 64;    // duration head width limit
constexpr int kMaxCluster = 4;
constexpr int kMaxFrames = 8;
constexpr int kMaxRows = 2 * kMaxFrames;  // frame rows of a window: up to two utterances x 8 frames

struct ScanArgs {
    const float* enc;      // (B, T, D)
    const float* pred;     // (B, D)
    const float* wt;       // (D, ldw): transposed joint weight, columns >= V ignored
    const float* wdur;     // (n_dur, D) or null
    const int32_t* in_lens;
    const int32_t* active;  // (n_active,) utterance indices, or null for 0..B-1
    int32_t* state;        // (B, 4): t, k (symbols at frame t), hyp_len, n_steps
    int64_t* prefix;       // (B, hyp_cap + 1): <sos> then the emitted tokens
    int32_t* durs;         // (B, dur_cap) or null
    int32_t* report;       // (B,): prefix length after an emission, 0 finished, -1 error
    int B, T, D, V, ldw, n_dur, blank, max_symbols, hyp_cap, dur_cap;
    int max_windows;  // windows one utterance may scan in this launch (0: no limit)
    int n_active;     // entries of `active`
    int stages;       // weight ring stages (kStageBytes each)
};

// a beats b under torch.argmax: NaN is the maximum, ties go to the lower index.
__device__ __forceinline__ bool beats(float a, int ai, float b, int bi) {
    const bool an = a != a, bn = b != b;
    if (an || bn) return an && (!bn || ai < bi);
    return a > b || (a == b && ai < bi);
}

__device__ __forceinline__ void warp_argmax(float& v, int& i) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, i, o);
        if (beats(ov, oi, v, i)) {
            v = ov;
            i = oi;
        }
    }
}


__device__ __forceinline__ void st_cluster_pair(uint32_t addr, float v, int i) {
    asm volatile("st.shared::cluster.v2.b32 [%0], {%1, %2};" ::"r"(addr), "r"(__float_as_uint(v)), "r"(i)
                 : "memory");
}

// ------------------------------------------------ joint weight stream
//
// The window's pass over the transposed joint weight is a per-thread cp.async
// pipeline: every thread copies its own CPT columns of the next rows into a
// private part of a shared-memory ring of `stages` 16 KB stages and later reads
// back only what it copied, so no CTA barrier is needed. Each weight row feeds
// only NF frames, so the stream runs at the L2 rate only with deep lookahead:
// the ring takes the shared memory the hidden rows leave (up to kMaxRingStages,
// one CTA per SM), keeping (stages - 1) stages of reads in flight.
constexpr int kMaxRingStages = 6;
constexpr int kMinRingStages = 2;
constexpr int kStageBytes = 16 * 1024;
constexpr size_t kScanSmemBudget = 110 * 1024;  // two CTAs per SM

template <int CPT>
struct Ring {
    static constexpr int kVec = CPT;                       // floats per copy (one per row and thread)
    static constexpr int kRows = kStageBytes / (4 * CPT * kScanThreads);  // weight rows per stage
    static constexpr int kStageFloats = kRows * CPT * kScanThreads;
};

template <int N>
__device__ __forceinline__ void cp_async(float* dst, const float* src, bool ok) {
    const uint32_t d = tc::smem_u32(dst);
    const int n = ok ? 4 * N : 0;  // 0: zero-fill, nothing read
    if constexpr (N == 4)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(n) : "memory");
    else if constexpr (N == 2)
        asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(d), "l"(src), "r"(n) : "memory");
    else
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(d), "l"(src), "r"(n) : "memory");
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// cp.async.wait_group takes an immediate: dispatch the (uniform) runtime count.
__device__ __forceinline__ void cp_async_wait_n(int n) {
    switch (n) {
        case 0: cp_async_wait<0>(); break;
        case 1: cp_async_wait<1>(); break;
        case 2: cp_async_wait<2>(); break;
        case 3: cp_async_wait<3>(); break;
        case 4: cp_async_wait<4>(); break;
        case 5: cp_async_wait<5>(); break;
        case 6: cp_async_wait<6>(); break;
        case 7: cp_async_wait<7>(); break;
        case 8: cp_async_wait<8>(); break;
        default: cp_async_wait<9>(); break;
    }
}

// Issues this thread's copies of weight rows [chunk * kRows, +kRows) into ring slot chunk % stages.
template <int CPT>
__device__ __forceinline__ void issue_chunk(float* ring, int stages, int chunk, int D, const float* wt, int ldw,
                                            int col, int tid) {
    using R = Ring<CPT>;
    float* base = ring + (size_t)(chunk % stages) * R::kStageFloats;
    const int j0 = chunk * R::kRows;
#pragma unroll
    for (int r = 0; r < R::kRows; ++r) {
        const int j = j0 + r;
        if (j < D) {
            const bool ok = col < ldw;
            cp_async<R::kVec>(base + ((size_t)r * kScanThreads + tid) * R::kVec, wt + (size_t)j * ldw + (ok ? col : 0),
                              ok);
        }
    }
    cp_async_commit();
}

template <int C, int NF, int RU>
__global__ void __launch_bounds__(kScanThreads, 2) greedy_scan_kernel(ScanArgs a) {
    static_assert(RU == 1 || C == 1, "utterance pairs run without clusters");
    constexpr int CPT = 4 / C;                        // consecutive vocab columns per thread and pass
    constexpr int kPass = CPT * kScanThreads;
    constexpr int NR = RU * NF;                       // frame rows per window: RU utterances x NF frames
    using R = Ring<CPT>;
    extern __shared__ __align__(16) float smem[];
    float* ring = smem;                                     // per-thread weight stream stages
    float* hs = smem + (size_t)a.stages * R::kStageFloats;  // RU x (D, NF): hidden rows, frame-minor
    float* ps = hs + (size_t)RU * a.D * NF;                 // RU x (D,): predictor outputs
    __shared__ float red_v[kMaxRows][kScanWarps];
    __shared__ int red_i[kMaxRows][kScanWarps];
    __shared__ __align__(8) int2 cand[2][kMaxCluster][kMaxRows];  // (value bits, index) per rank
    __shared__ float dur_v[kMaxRows][kMaxScanDur];
    __shared__ int best_tok[kMaxRows], best_dur[kMaxRows];
    __shared__ int s_t[RU], s_k[RU], s_len[RU], s_steps[RU], s_go[RU], s_t0[RU], s_nf[RU];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int rank = C > 1 ? (int)tc::cluster_ctarank() : 0;
    const int slot0 = (blockIdx.x / C) * RU;
    const int n_slots = a.active ? a.n_active : a.B;
    int bs[RU], Tbs[RU];
#pragma unroll
    for (int r = 0; r < RU; ++r) {
        const int sl = slot0 + r;
        bs[r] = sl < n_slots ? (a.active ? a.active[sl] : sl) : -1;
        Tbs[r] = bs[r] >= 0 ? min(max(a.in_lens[bs[r]], 0), a.T) : 0;
    }
    if (tid < RU) {
        const int r = tid;
        if (bs[r] >= 0) {
            const int32_t* st = a.state + 4 * bs[r];
            s_t[r] = st[0];
            s_k[r] = st[1];
            s_len[r] = st[2];
            s_steps[r] = st[3];
            if (a.max_symbols <= 0) s_t[r] = Tbs[r];  // the reference's per-frame loop never runs
            s_go[r] = s_t[r] < Tbs[r];
            if (!s_go[r] && rank == 0) {
                a.state[4 * bs[r]] = s_t[r];
                a.report[bs[r]] = 0;
            }
        } else {
            s_go[r] = 0;
        }
    }
#pragma unroll
    for (int r = 0; r < RU; ++r) {
        if (bs[r] < 0) continue;
        const float* pr = a.pred + (size_t)bs[r] * a.D;
        for (int j = tid; j < a.D; j += kScanThreads) ps[(size_t)r * a.D + j] = pr[j];
    }
    __syncthreads();
    bool any = false;
#pragma unroll
    for (int r = 0; r < RU; ++r) any |= s_go[r] != 0;
    if (!any) return;  // uniform over the cluster: every CTA read the same state
    const bool tdt = a.n_dur > 0;
    // This CTA's vocabulary slice [lo, hi).
    const int slice = ((a.V + C - 1) / C + 3) / 4 * 4;
    const int lo = rank * slice, hi = min(a.V, lo + slice);
    int parity = 0, windows = 0;

    for (;;) {
        if (tid < RU) {
            s_t0[tid] = s_t[tid];
            s_nf[tid] = s_go[tid] ? min(NF, Tbs[tid] - s_t[tid]) : 0;
        }
        __syncthreads();
        // Hidden rows of the window, frame-minor so one vector read serves all frames;
        // rows of a stopped utterance (or past its end) are zero.
#pragma unroll
        for (int r = 0; r < RU; ++r) {
            const int t0 = s_t0[r], nf = s_nf[r];
            const float* encb = a.enc + ((size_t)max(bs[r], 0) * a.T) * a.D;
            for (int j = tid; j < a.D; j += kScanThreads) {
                const float p = ps[(size_t)r * a.D + j];
                float hv[NF];
#pragma unroll
                for (int f = 0; f < NF; ++f) hv[f] = f < nf ? tanhf(encb[(size_t)(t0 + f) * a.D + j] + p) : 0.f;
                float4* dst = reinterpret_cast<float4*>(hs + ((size_t)r * a.D + j) * NF);
#pragma unroll
                for (int q = 0; q < NF / 4; ++q)
                    dst[q] = make_float4(hv[4 * q], hv[4 * q + 1], hv[4 * q + 2], hv[4 * q + 3]);
            }
        }
        __syncthreads();

        float bv[NR];
        int bi[NR];
#pragma unroll
        for (int f = 0; f < NR; ++f) {
            bv[f] = -INFINITY;
            bi[f] = INT_MAX;
        }
        for (int c0 = lo; c0 < hi; c0 += kPass) {
            const int col = c0 + CPT * tid;
            float acc[NR][CPT];
#pragma unroll
            for (int f = 0; f < NR; ++f)
#pragma unroll
                for (int c = 0; c < CPT; ++c) acc[f][c] = 0.f;
            // Lanes that stream weights (a partial last pass leaves some idle).
            const unsigned live = __ballot_sync(0xffffffffu, col < hi);
            if (col < hi) {
                const int nch = (a.D + R::kRows - 1) / R::kRows;
                for (int c = 0; c < a.stages - 1; ++c) {
                    if (c < nch)
                        issue_chunk<CPT>(ring, a.stages, c, a.D, a.wt, a.ldw, col, tid);
                    else
                        cp_async_commit();
                }
                for (int ch = 0; ch < nch; ++ch) {
                    const int nx = ch + a.stages - 1;
                    // The slot refilled now was read in the previous iteration: order those
                    // shared-memory reads before the asynchronous writes.
                    __syncwarp(live);
                    if (nx < nch)
                        issue_chunk<CPT>(ring, a.stages, nx, a.D, a.wt, a.ldw, col, tid);
                    else
                        cp_async_commit();
                    cp_async_wait_n(a.stages - 1);  // this thread's copies of chunk ch have landed
                    const float* base = ring + (size_t)(ch % a.stages) * R::kStageFloats;
#pragma unroll
                    for (int rr = 0; rr < R::kRows; ++rr) {
                        const int j = ch * R::kRows + rr;
                        if (j < a.D) {
                            float w[CPT];
                            const float* src = base + ((size_t)rr * kScanThreads + tid) * CPT;
                            if constexpr (CPT == 4) {
                                const float4 v = *reinterpret_cast<const float4*>(src);
                                w[0] = v.x, w[1] = v.y, w[2] = v.z, w[3] = v.w;
                            } else if constexpr (CPT == 2) {
                                const float2 v = *reinterpret_cast<const float2*>(src);
                                w[0] = v.x, w[1] = v.y;
                            } else {
                                w[0] = *src;
                            }
#pragma unroll
                            for (int r = 0; r < RU; ++r) {
                                float hf[NF];
#pragma unroll
                                for (int q = 0; q < NF / 4; ++q) {
                                    const float4 h =
                                        *reinterpret_cast<const float4*>(hs + ((size_t)r * a.D + j) * NF + 4 * q);
                                    hf[4 * q] = h.x, hf[4 * q + 1] = h.y, hf[4 * q + 2] = h.z, hf[4 * q + 3] = h.w;
                                }
#pragma unroll
                                for (int f = 0; f < NF; ++f)
#pragma unroll
                                    for (int c = 0; c < CPT; ++c)
                                        acc[r * NF + f][c] = fmaf(w[c], hf[f], acc[r * NF + f][c]);
                            }
                        }
                    }
                }
                cp_async_wait<0>();
            }
#pragma unroll
            for (int f = 0; f < NR; ++f)
#pragma unroll
                for (int c = 0; c < CPT; ++c) {
                    const int cc = col + c;
                    if (cc < hi && beats(acc[f][c], cc, bv[f], bi[f])) {
                        bv[f] = acc[f][c];
                        bi[f] = cc;
                    }
                }
        }
#pragma unroll
        for (int f = 0; f < NR; ++f) {
            warp_argmax(bv[f], bi[f]);
            if (lane == 0) {
                red_v[f][warp] = bv[f];
                red_i[f][warp] = bi[f];
            }
        }
        // Duration head (every CTA, a few columns): warp w owns columns w, w + 8, ...
        if (tdt) {
            for (int c = warp; c < a.n_dur; c += kScanWarps) {
                const float* wd = a.wdur + (size_t)c * a.D;
                float sd[NR];
#pragma unroll
                for (int f = 0; f < NR; ++f) sd[f] = 0.f;
                for (int j = lane; j < a.D; j += 32) {
                    const float w = __ldg(wd + j);
#pragma unroll
                    for (int r = 0; r < RU; ++r)
#pragma unroll
                        for (int q = 0; q < NF / 4; ++q) {
                            const float4 h = *reinterpret_cast<const float4*>(hs + ((size_t)r * a.D + j) * NF + 4 * q);
                            const int f0 = r * NF + 4 * q;
                            sd[f0] = fmaf(w, h.x, sd[f0]);
                            sd[f0 + 1] = fmaf(w, h.y, sd[f0 + 1]);
                            sd[f0 + 2] = fmaf(w, h.z, sd[f0 + 2]);
                            sd[f0 + 3] = fmaf(w, h.w, sd[f0 + 3]);
                        }
                }
#pragma unroll
                for (int f = 0; f < NR; ++f) {
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) sd[f] += __shfl_xor_sync(0xffffffffu, sd[f], o);
                    if (lane == 0) dur_v[f][c] = sd[f];
                }
            }
        }
        __syncthreads();
        if (tid < NR) {
            float v = red_v[tid][0];
            int i = red_i[tid][0];
            for (int w = 1; w < kScanWarps; ++w)
                if (beats(red_v[tid][w], red_i[tid][w], v, i)) {
                    v = red_v[tid][w];
                    i = red_i[tid][w];
                }
            if constexpr (C > 1) {
                const uint32_t local = tc::smem_u32(&cand[parity][rank][tid]);
#pragma unroll
                for (int r = 0; r < C; ++r) st_cluster_pair(tc::mapa_shared(local, r), v, i);
            } else {
                best_tok[tid] = i;
            }
            if (tdt) {
                float dv = dur_v[tid][0];
                int di = 0;
                for (int c = 1; c < a.n_dur; ++c)
                    if (beats(dur_v[tid][c], c, dv, di)) {
                        dv = dur_v[tid][c];
                        di = c;
                    }
                best_dur[tid] = di;  // durations are range(max_duration + 1): index == value
            }
        }
        if constexpr (C > 1) {
            tc::cluster_sync();  // candidates of every rank have landed in every CTA
            if (tid < NR) {
                float v = __int_as_float(cand[parity][0][tid].x);
                int i = cand[parity][0][tid].y;
#pragma unroll
                for (int r = 1; r < C; ++r) {
                    const float rv = __int_as_float(cand[parity][r][tid].x);
                    const int ri = cand[parity][r][tid].y;
                    if (beats(rv, ri, v, i)) {
                        v = rv;
                        i = ri;
                    }
                }
                best_tok[tid] = i;
            }
            parity ^= 1;
        }
        __syncthreads();

        // The reference state machine over the window: thread 32 r walks utterance r
        // (identical in every CTA of a cluster; rank 0 writes the outputs).
        ++windows;
        if ((tid & 31) == 0 && (tid >> 5) < RU && s_go[tid >> 5]) {
            const int r = tid >> 5;
            const int b = bs[r], Tb = Tbs[r];
            const int t0 = s_t0[r], nf = s_nf[r];
            const int* btok = best_tok + r * NF;
            const int* bdur = best_dur + r * NF;
            const bool out = rank == 0;
            int t = t0, k = s_k[r], len = s_len[r], steps = s_steps[r];
            int emitted = 0, err = 0;
            int64_t* pre = a.prefix + (size_t)b * (a.hyp_cap + 1);
            while (t < t0 + nf) {
                const int tok = btok[t - t0];
                if (!tdt) {
                    if (tok == a.blank) {  // rnnt.py:31-32
                        ++t;
                        k = 0;
                        continue;
                    }
                    if (len >= a.hyp_cap) {
                        err = 1;
                        break;
                    }
                    if (out) pre[1 + len] = tok;
                    ++len;
                    emitted = 1;
                    if (++k >= a.max_symbols) {  // rnnt.py:29 loop exhausted: next frame
                        ++t;
                        k = 0;
                    }
                    break;
                }
                const int dv = bdur[t - t0];
                if (steps >= a.dur_cap) {
                    err = 1;
                    break;
                }
                if (out) a.durs[(size_t)b * a.dur_cap + steps] = dv;  // tdt.py:45
                ++steps;
                if (tok != a.blank) {  // tdt.py:46-49
                    if (len >= a.hyp_cap) {
                        err = 1;
                        break;
                    }
                    if (out) pre[1 + len] = tok;
                    ++len;
                    emitted = 1;
                }
                if (dv > 0) {  // tdt.py:50-52
                    t += dv;
                    k = 0;
                } else if (tok == a.blank) {  // tdt.py:54-56
                    ++t;
                    k = 0;
                } else if (++k >= a.max_symbols) {  // tdt.py:57-59
                    ++t;
                    k = 0;
                }
                if (emitted) break;
            }
            s_t[r] = t;
            s_k[r] = k;
            s_len[r] = len;
            s_steps[r] = steps;
            const bool finished = err || emitted || t >= Tb;
            // A long run of blanks is continued by the next launch: the launch's
            // duration is set by its longest chain of windows.
            const bool paused = !finished && a.max_windows > 0 && windows >= a.max_windows;
            s_go[r] = !(finished || paused);
            if ((finished || paused) && out) {
                int32_t* st = a.state + 4 * b;
                st[0] = t;
                st[1] = k;
                st[2] = len;
                st[3] = steps;
                a.report[b] = err ? -1 : (emitted ? len + 1 : (paused ? -2 : 0));
            }
        }
        __syncthreads();
        bool more = false;
#pragma unroll
        for (int r = 0; r < RU; ++r) more |= s_go[r] != 0;
        if (!more) return;  // every CTA of the cluster stops after the same window
    }
}

__global__ void pack_weights_kernel(const float* __restrict__ W, int V, int D, float* __restrict__ wt, int ldw) {
    __shared__ float tile[32][33];
    const int v0 = blockIdx.x * 32, j0 = blockIdx.y * 32;
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        const int v = v0 + r, j = j0 + threadIdx.x;
        tile[r][threadIdx.x] = (v < V && j < D) ? W[(size_t)v * D + j] : 0.f;
    }
    __syncthreads();
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        const int j = j0 + r, v = v0 + threadIdx.x;
        if (j < D && v < ldw) wt[(size_t)j * ldw + v] = tile[threadIdx.x][r];
    }
}

// Zeroes the state and fills every prefix position with <sos>: position 0 is the
// reference's start token, and positions past a hypothesis then hold a valid token
// id for predictors that are run on right-padded prefixes.
__global__ void greedy_init_kernel(int32_t* state, int64_t* prefix, int B, int hyp_cap, int sos) {
    const size_t n = (size_t)B * (hyp_cap + 1), ns = 4 * (size_t)B;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n || i < ns; i += (size_t)gridDim.x * blockDim.x) {
        if (i < n) prefix[i] = sos;
        if (i < ns) state[i] = 0;
    }
}

using ScanKernel = void (*)(ScanArgs);

template <int C, int NF, int RU>
int launch_scan(const ScanArgs& a, int n_ctas, size_t smem, cudaStream_t stream) {
    ScanKernel k = greedy_scan_kernel<C, NF, RU>;
    if (smem > 48 * 1024)
        ASR_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(n_ctas * C);
    cfg.blockDim = dim3(kScanThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = C;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = C > 1 ? 1 : 0;
    ASR_CUDA_TRY(cudaLaunchKernelEx(&cfg, k, a));
    return ASR_OK;
}

template <int NF>
int launch_scan_c(int C, int RU, const ScanArgs& a, int n_slots, size_t smem, cudaStream_t stream) {
    if (RU == 2) return launch_scan<1, NF, 2>(a, (n_slots + 1) / 2, smem, stream);
    switch (C) {
        case 1: return launch_scan<1, NF, 1>(a, n_slots, smem, stream);
        case 2: return launch_scan<2, NF, 1>(a, n_slots, smem, stream);
        default: return launch_scan<4, NF, 1>(a, n_slots, smem, stream);
    }
}

int env_choice(const char* name, int fallback) {
    const char* e = std::getenv(name);
    return e ? std::atoi(e) : fallback;
}

}  // namespace
}  // namespace asr

using namespace asr;

extern "C" int asr_greedy_pack_weights(const float* joint_W, int V, int d, float* joint_Wt, int ldw,
                                       asr_stream_t stream) {
    if (V < 1 || d < 1 || ldw < V || ldw % 4 != 0 || !joint_W || !joint_Wt) return ASR_ERR_INVALID_ARGUMENT;
    if (reinterpret_cast<uintptr_t>(joint_Wt) % 16 != 0) return ASR_ERR_INVALID_ARGUMENT;
    KernelTimer kt("greedy_pack", stream);
    const dim3 grid((ldw + 31) / 32, (d + 31) / 32);
    pack_weights_kernel<<<grid, dim3(32, 8), 0, stream>>>(joint_W, V, d, joint_Wt, ldw);
    ASR_LAUNCH_CHECK();
    return ASR_OK;
}

extern "C" int asr_greedy_init(int32_t* state, int64_t* prefix, int B, int hyp_cap, int sos_id,
                               asr_stream_t stream) {
    if (B < 0 || hyp_cap < 0) return ASR_ERR_INVALID_ARGUMENT;
    if (B == 0) return ASR_OK;
    if (!state || !prefix) return ASR_ERR_INVALID_ARGUMENT;
    KernelTimer kt("greedy_init", stream);
    const size_t n = std::max((size_t)B * (hyp_cap + 1), 4 * (size_t)B);
    const int grid = (int)std::min<size_t>((n + 255) / 256, (size_t)sm_count() * 8);
    greedy_init_kernel<<<grid, 256, 0, stream>>>(state, prefix, B, hyp_cap, sos_id);
    ASR_LAUNCH_CHECK();
    return ASR_OK;
}


extern "C" int asr_greedy_scan(const float* encoder, const float* pred, const float* joint_Wt, int ldw,
                               const float* joint_W_dur, const int32_t* in_lens, const int32_t* active,
                               int n_active, int32_t* state, int64_t* prefix, int32_t* durs, int32_t* report, int B,
                               int T, int d, int V, int n_dur, int blank_idx, int max_symbols, int hyp_cap,
                               int dur_cap, int max_windows, asr_stream_t stream) {
    if (B < 0 || T < 1 || d < 1 || V < 1 || n_dur < 0 || hyp_cap < 0 || dur_cap < 0) return ASR_ERR_INVALID_ARGUMENT;
    if (ldw < V || ldw % 4 != 0 || blank_idx < 0 || blank_idx >= V || max_windows < 0) return ASR_ERR_INVALID_ARGUMENT;
    const int n_slots = active ? n_active : B;
    if (n_slots < 0 || n_slots > B) return ASR_ERR_INVALID_ARGUMENT;
    if (n_slots == 0) return ASR_OK;
    if (!encoder || !pred || !joint_Wt || !in_lens || !state || !prefix || !report) return ASR_ERR_INVALID_ARGUMENT;
    if (n_dur > 0 && (!joint_W_dur || !durs)) return ASR_ERR_INVALID_ARGUMENT;
    if (reinterpret_cast<uintptr_t>(joint_Wt) % 16 != 0) return ASR_ERR_INVALID_ARGUMENT;
    if (d > kMaxScanDim || n_dur > kMaxScanDur) return ASR_ERR_UNSUPPORTED;
    ScanArgs a{encoder, pred, joint_Wt, joint_W_dur, in_lens, active, state, prefix, durs, report,
               B, T, d, V, ldw, n_dur, blank_idx, max_symbols, hyp_cap, dur_cap, max_windows, 0, 0};
    // Cluster width: one CTA per utterance while the active utterances fill the
    // GPU; otherwise split the vocabulary over up to kMaxCluster SMs per utterance.
    static const int env_c = env_choice("ASR_B200_DECODE_CLUSTER", 0);
    static const int env_f = env_choice("ASR_B200_DECODE_FRAMES", 0);
    static const int env_p = env_choice("ASR_B200_DECODE_PAIRS", -1);
    const int sms = sm_count();
    int C = 1;
    if (env_c == 1 || env_c == 2 || env_c == 4) {
        C = env_c;
    } else if (V >= 512) {
        while (C < kMaxCluster && n_slots * C * 2 <= sms) C *= 2;
    }
    // Two utterances per CTA (one pass over the weight for both) halve the L2
    // weight stream but measured slower on B200 (scan 41.4 vs 36.2 ms at config-5
    // shapes): the saturated launches are issue-bound, not L2-bound. Opt-in only
    // (ASR_B200_DECODE_PAIRS=1).
    const int RU = (env_p == 1 && C == 1) ? 2 : 1;
    a.n_active = n_slots;
    const int NF = env_f == 4 ? 4 : 8;
    // Shared memory: hidden rows + predictor rows, the rest of the budget for the ring.
    const size_t rows = sizeof(float) * (size_t)RU * d * (NF + 1);
    const int stages = rows + kMinRingStages * kStageBytes > kScanSmemBudget
                           ? kMinRingStages
                           : (int)std::min<size_t>(kMaxRingStages, (kScanSmemBudget - rows) / kStageBytes);
    if (stages < kMinRingStages) return ASR_ERR_UNSUPPORTED;
    a.stages = stages;
    const size_t smem = rows + (size_t)stages * kStageBytes;
    KernelTimer kt("greedy_scan", stream);
    return NF == 4 ? launch_scan_c<4>(C, RU, a, n_slots, smem, stream)
                   : launch_scan_c<8>(C, RU, a, n_slots, smem, stream);
}
