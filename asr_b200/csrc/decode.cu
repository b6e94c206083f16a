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
// of greedy_scan_kernel therefore advances EVERY active utterance (one CTA
// each) from its current state to its next emitted token or to its end:
//   * the hidden rows tanh(enc[b, t..t+kWin) + pred) of a window of frames are
//     built in shared memory (the joint row is never written to HBM);
//   * the window's logits come from one pass over the transposed joint weight
//     (L2-resident, read once per window and reused for all kWin frames from
//     registers), each thread owning 8 vocab columns x kWin frames;
//   * the first maximal index per frame (torch.argmax semantics; NaN counts as
//     the maximum) is reduced across the CTA, the duration head likewise;
//   * one thread then replays the reference's state machine over the window
//     (blank advances a frame, TDT durations jump frames, max_symbols_per_frame
//     forces progress), recording every TDT duration, until a token is emitted
//     (the host must run the predictor) or the utterance ends. Frames past the
//     stopping point were computed speculatively and are discarded.
// The host loop (asr_b200/decode) thus runs one launch per emitted-token level
// instead of one joint call per step and utterance.
#include <climits>

#include "common.cuh"

namespace asr {
namespace {

constexpr int kWin = 8;                                   // frames per window
constexpr int kScanThreads = 128;                         // 4 warps
constexpr int kScanWarps = kScanThreads / 32;
constexpr int kColTile = kScanThreads * 8;                // vocab columns per pass
constexpr int kMaxScanDim = 4096;                         // joint dim limit (shared memory)
constexpr int kMaxScanDur = 64;                           // duration head width limit

struct ScanArgs {
    const float* enc;     // (B, T, D)
    const float* pred;    // (B, D)
    const float* wt;      // (D, ldw): transposed joint weight, columns >= V ignored
    const float* wdur;    // (n_dur, D) or null
    const int32_t* in_lens;
    int32_t* state;       // (B, 4): t, k (symbols at frame t), hyp_len, n_steps
    int64_t* prefix;      // (B, hyp_cap + 1): <sos> then the emitted tokens
    int32_t* durs;        // (B, dur_cap) or null
    int32_t* report;      // (B,): prefix length after an emission, 0 finished, -1 error
    int B, T, D, V, ldw, n_dur, blank, max_symbols, hyp_cap, dur_cap;
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

__device__ __forceinline__ void fma4(float (&acc)[8], const float4 w, const float h, const int base) {
    acc[base + 0] = fmaf(w.x, h, acc[base + 0]);
    acc[base + 1] = fmaf(w.y, h, acc[base + 1]);
    acc[base + 2] = fmaf(w.z, h, acc[base + 2]);
    acc[base + 3] = fmaf(w.w, h, acc[base + 3]);
}

__global__ void __launch_bounds__(kScanThreads) greedy_scan_kernel(ScanArgs a) {
    extern __shared__ __align__(16) float smem[];
    float* hs = smem;                       // (D, kWin): hidden rows, frame-minor
    float* ps = smem + (size_t)a.D * kWin;  // (D,): predictor output
    __shared__ float red_v[kWin][kScanWarps];
    __shared__ int red_i[kWin][kScanWarps];
    __shared__ float dur_v[kWin][kMaxScanDur];
    __shared__ int best_tok[kWin], best_dur[kWin];
    __shared__ int s_t, s_k, s_len, s_steps, s_go;

    const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int Tb = min(max(a.in_lens[b], 0), a.T);
    int32_t* st = a.state + 4 * b;
    if (tid == 0) {
        s_t = st[0];
        s_k = st[1];
        s_len = st[2];
        s_steps = st[3];
        if (a.max_symbols <= 0) s_t = Tb;  // the reference's per-frame loop never runs
    }
    const float* pr = a.pred + (size_t)b * a.D;
    for (int j = tid; j < a.D; j += kScanThreads) ps[j] = pr[j];
    __syncthreads();
    if (s_t >= Tb) {
        if (tid == 0) {
            st[0] = s_t;
            a.report[b] = 0;
        }
        return;
    }
    const float* encb = a.enc + (size_t)b * a.T * a.D;
    const bool tdt = a.n_dur > 0;

    for (;;) {
        const int t0 = s_t;
        const int nf = min(kWin, Tb - t0);
        // Hidden rows of the window, frame-minor so one 32-byte read serves all frames.
        for (int j = tid; j < a.D; j += kScanThreads) {
            const float p = ps[j];
            float hv[kWin];
#pragma unroll
            for (int f = 0; f < kWin; ++f) hv[f] = f < nf ? tanhf(encb[(size_t)(t0 + f) * a.D + j] + p) : 0.f;
            float4* dst = reinterpret_cast<float4*>(hs + (size_t)j * kWin);
            dst[0] = make_float4(hv[0], hv[1], hv[2], hv[3]);
            dst[1] = make_float4(hv[4], hv[5], hv[6], hv[7]);
        }
        __syncthreads();

        float bv[kWin];
        int bi[kWin];
#pragma unroll
        for (int f = 0; f < kWin; ++f) {
            bv[f] = -INFINITY;
            bi[f] = INT_MAX;
        }
        for (int c0 = 0; c0 < a.V; c0 += kColTile) {
            const int ca = c0 + 4 * tid, cb = ca + 4 * kScanThreads;
            const bool va = ca < a.ldw, vb = cb < a.ldw;
            float acc[kWin][8];
#pragma unroll
            for (int f = 0; f < kWin; ++f)
#pragma unroll
                for (int c = 0; c < 8; ++c) acc[f][c] = 0.f;
            const float* wa = a.wt + ca;
            const float* wb = a.wt + cb;
#pragma unroll 4
            for (int j = 0; j < a.D; ++j) {
                const size_t row = (size_t)j * a.ldw;
                const float4 w0 = va ? __ldg(reinterpret_cast<const float4*>(wa + row)) : make_float4(0, 0, 0, 0);
                const float4 w1 = vb ? __ldg(reinterpret_cast<const float4*>(wb + row)) : make_float4(0, 0, 0, 0);
                const float4 h0 = *reinterpret_cast<const float4*>(hs + (size_t)j * kWin);
                const float4 h1 = *reinterpret_cast<const float4*>(hs + (size_t)j * kWin + 4);
                const float hf[kWin] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
#pragma unroll
                for (int f = 0; f < kWin; ++f) {
                    fma4(acc[f], w0, hf[f], 0);
                    fma4(acc[f], w1, hf[f], 4);
                }
            }
#pragma unroll
            for (int f = 0; f < kWin; ++f)
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    const int col = (c < 4 ? ca : cb) + (c & 3);
                    if (col < a.V && beats(acc[f][c], col, bv[f], bi[f])) {
                        bv[f] = acc[f][c];
                        bi[f] = col;
                    }
                }
        }
#pragma unroll
        for (int f = 0; f < kWin; ++f) {
            warp_argmax(bv[f], bi[f]);
            if (lane == 0) {
                red_v[f][warp] = bv[f];
                red_i[f][warp] = bi[f];
            }
        }
        // Duration head: warp w owns columns w, w + 4, ...; lanes split the joint dim.
        if (tdt) {
            for (int c = warp; c < a.n_dur; c += kScanWarps) {
                const float* wd = a.wdur + (size_t)c * a.D;
                float s[kWin];
#pragma unroll
                for (int f = 0; f < kWin; ++f) s[f] = 0.f;
                for (int j = lane; j < a.D; j += 32) {
                    const float w = __ldg(wd + j);
                    const float4 h0 = *reinterpret_cast<const float4*>(hs + (size_t)j * kWin);
                    const float4 h1 = *reinterpret_cast<const float4*>(hs + (size_t)j * kWin + 4);
                    s[0] = fmaf(w, h0.x, s[0]);
                    s[1] = fmaf(w, h0.y, s[1]);
                    s[2] = fmaf(w, h0.z, s[2]);
                    s[3] = fmaf(w, h0.w, s[3]);
                    s[4] = fmaf(w, h1.x, s[4]);
                    s[5] = fmaf(w, h1.y, s[5]);
                    s[6] = fmaf(w, h1.z, s[6]);
                    s[7] = fmaf(w, h1.w, s[7]);
                }
#pragma unroll
                for (int f = 0; f < kWin; ++f) {
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) s[f] += __shfl_xor_sync(0xffffffffu, s[f], o);
                    if (lane == 0) dur_v[f][c] = s[f];
                }
            }
        }
        __syncthreads();
        if (tid < kWin) {
            float v = red_v[tid][0];
            int i = red_i[tid][0];
            for (int w = 1; w < kScanWarps; ++w)
                if (beats(red_v[tid][w], red_i[tid][w], v, i)) {
                    v = red_v[tid][w];
                    i = red_i[tid][w];
                }
            best_tok[tid] = i;
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
        __syncthreads();

        // The reference state machine over the window (one thread; a few steps).
        if (tid == 0) {
            int t = t0, k = s_k, len = s_len, steps = s_steps;
            int emitted = 0, err = 0;
            int64_t* pre = a.prefix + (size_t)b * (a.hyp_cap + 1);
            while (t < t0 + nf) {
                const int tok = best_tok[t - t0];
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
                    pre[1 + len++] = tok;
                    emitted = 1;
                    if (++k >= a.max_symbols) {  // rnnt.py:29 loop exhausted: next frame
                        ++t;
                        k = 0;
                    }
                    break;
                }
                const int dv = best_dur[t - t0];
                if (steps >= a.dur_cap) {
                    err = 1;
                    break;
                }
                a.durs[(size_t)b * a.dur_cap + steps++] = dv;  // tdt.py:45
                if (tok != a.blank) {                          // tdt.py:46-49
                    if (len >= a.hyp_cap) {
                        err = 1;
                        break;
                    }
                    pre[1 + len++] = tok;
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
            s_t = t;
            s_k = k;
            s_len = len;
            s_steps = steps;
            const int done = err || emitted || t >= Tb;
            s_go = !done;
            if (done) {
                st[0] = t;
                st[1] = k;
                st[2] = len;
                st[3] = steps;
                a.report[b] = err ? -1 : (emitted ? len + 1 : 0);
            }
        }
        __syncthreads();
        if (!s_go) return;
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

__global__ void greedy_init_kernel(int32_t* state, int64_t* prefix, int B, int hyp_cap, int sos) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    for (int i = 0; i < 4; ++i) state[4 * b + i] = 0;
    prefix[(size_t)b * (hyp_cap + 1)] = sos;
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
    greedy_init_kernel<<<(B + 127) / 128, 128, 0, stream>>>(state, prefix, B, hyp_cap, sos_id);
    ASR_LAUNCH_CHECK();
    return ASR_OK;
}

extern "C" int asr_greedy_scan(const float* encoder, const float* pred, const float* joint_Wt, int ldw,
                               const float* joint_W_dur, const int32_t* in_lens, int32_t* state, int64_t* prefix,
                               int32_t* durs, int32_t* report, int B, int T, int d, int V, int n_dur,
                               int blank_idx, int max_symbols, int hyp_cap, int dur_cap, asr_stream_t stream) {
    if (B < 0 || T < 1 || d < 1 || V < 1 || n_dur < 0 || hyp_cap < 0 || dur_cap < 0) return ASR_ERR_INVALID_ARGUMENT;
    if (ldw < V || ldw % 4 != 0 || blank_idx < 0 || blank_idx >= V) return ASR_ERR_INVALID_ARGUMENT;
    if (B == 0) return ASR_OK;
    if (!encoder || !pred || !joint_Wt || !in_lens || !state || !prefix || !report) return ASR_ERR_INVALID_ARGUMENT;
    if (n_dur > 0 && (!joint_W_dur || !durs)) return ASR_ERR_INVALID_ARGUMENT;
    if (reinterpret_cast<uintptr_t>(joint_Wt) % 16 != 0) return ASR_ERR_INVALID_ARGUMENT;
    if (d > kMaxScanDim || n_dur > kMaxScanDur) return ASR_ERR_UNSUPPORTED;
    ScanArgs a{encoder, pred, joint_Wt, joint_W_dur, in_lens, state, prefix, durs, report,
               B, T, d, V, ldw, n_dur, blank_idx, max_symbols, hyp_cap, dur_cap};
    const size_t smem = sizeof(float) * (size_t)d * (kWin + 1);
    if (smem > 48 * 1024)
        ASR_CUDA_TRY(cudaFuncSetAttribute(greedy_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    KernelTimer kt("greedy_scan", stream);
    greedy_scan_kernel<<<B, kScanThreads, smem, stream>>>(a);
    ASR_LAUNCH_CHECK();
    return ASR_OK;
}
