// CTC prefix beam search on the GPU: one CTA per utterance. Replaces the
// reference's CPU op asr::beam_decode (src/asr/decode/csrc/ctc.cpp:46-137, a trie
// of prefixes and a hash map of next-beam entries per frame, OpenMP over the
// batch) with the same search:
//   for every frame t < in_len, every beam entry (prefix, p_blank, p_nonblank)
//   and every token v: v = blank keeps the prefix (p_blank += total + lp[v]); v =
//   the prefix's last token keeps the prefix from p_nonblank and extends it from
//   p_blank; any other v extends it from total; the beam_width candidates of
//   highest total = p_blank (+) p_nonblank survive (+ = logaddexp, float32).
//
// Per frame, on the CTA:
//   1. the frame's top (W + 1) non-blank tokens by log-prob (a block-wide radix
//      select over the row in shared memory). Only extensions by these tokens can survive: every
//      other extension of an entry is beaten by at least W extensions of the same
//      entry (same base score, larger log-prob, distinct prefixes), so the search
//      keeps exactly the reference's candidates while scoring W (W + 2) of them
//      instead of W x V;
//   2. "stay" candidates (an entry keeping its prefix). A prefix reachable both by
//      staying and by extending its parent (also in the beam) is one candidate:
//      the parent's extension score is added into the stay, and the duplicate
//      extension is dropped. Prefix identity uses a 64-bit polynomial hash of the
//      token sequence plus its length, so prefixes that left the beam and came
//      back still merge (the reference's trie nodes give the same identity);
//   3. the W best candidates (the same radix select); new prefixes get a
//      node (parent, token) in the utterance's node pool for the final backtrack.
// Ties between equal scores resolve by candidate order (the reference's
// nth_element leaves them unspecified).
#include <algorithm>
#include <climits>

#include "common.cuh"

namespace asr {
namespace {

constexpr int kBeamThreads = 256;
constexpr int kMaxBeam = 64;
constexpr int kMaxBeamVocab = 8192;
constexpr unsigned long long kHashMul = 0x100000001B3ull;  // odd multiplier of the prefix hash

// logaddexp as the reference computes it (ctc.cpp:28-34), in float32.
__device__ __forceinline__ int lane_of(int tid) { return tid & 31; }

__device__ __forceinline__ float lae_ref(float a, float b) {
    if (a == -INFINITY) return b;
    if (b == -INFINITY) return a;
    const float hi = fmaxf(a, b), lo = fminf(a, b);
    return hi + log1pf(expf(lo - hi));
}

// a sorts before b: valid entries (val >= 0) first, then larger key, then smaller val.
__device__ __forceinline__ bool before(float ka, int va, float kb, int vb) {
    if ((va >= 0) != (vb >= 0)) return va >= 0;
    if (ka != kb) return ka > kb;
    return va < vb;
}

// Order-preserving image of a float score (larger float -> larger unsigned).
__device__ __forceinline__ unsigned key_bits(float x) {
    const unsigned u = __float_as_uint(x);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// The K first pairs in `before` order of the n (key, val) pairs in shared memory
// (val < 0 marks an invalid pair; n_valid of them are valid), written sorted to
// okey / oval; returns how many (min(K, n_valid)). A radix select on key_bits, one
// 8-bit digit per pass (four passes at most, double-buffered histograms), finds the
// K-th score; pairs above it are taken, pairs equal to it in index order; then one
// warp sorts the <= kSelMax winners with shuffles. All threads call it; it ends with
// a barrier.
constexpr int kSelMax = 128;

struct SelScratch {
    int hist[2][256];
    int warp_cnt[kBeamThreads / 32];
    int digit, above, n_out;
};

// Sorts the k <= 32 E (key, val) pairs at key / val into `before` order: one warp,
// E pairs per lane, a bitonic network over shuffles.
template <int E>
__device__ void warp_sort(float* key, int* val, int k) {
    constexpr int N = 32 * E;
    const int lane = threadIdx.x & 31;
    float kk[E];
    int vv[E];
#pragma unroll
    for (int e = 0; e < E; ++e) {
        const int i = lane * E + e;
        kk[e] = i < k ? key[i] : -INFINITY;
        vv[e] = i < k ? val[i] : -1;
    }
#pragma unroll
    for (int ks = 2; ks <= N; ks <<= 1) {
#pragma unroll
        for (int j = ks >> 1; j > 0; j >>= 1) {
            if (j < E) {  // both elements in this lane
#pragma unroll
                for (int e = 0; e < E; ++e) {
                    const int p = e ^ j;
                    if (p > e) {
                        const int i = lane * E + e;
                        const bool fwd = (i & ks) == 0;
                        const bool sw = fwd ? before(kk[p], vv[p], kk[e], vv[e]) : before(kk[e], vv[e], kk[p], vv[p]);
                        if (sw) {
                            const float tk = kk[e];
                            kk[e] = kk[p];
                            kk[p] = tk;
                            const int tv = vv[e];
                            vv[e] = vv[p];
                            vv[p] = tv;
                        }
                    }
                }
            } else {  // the partner element sits in lane ^ (j / E), same slot
                const int lm = j / E;
#pragma unroll
                for (int e = 0; e < E; ++e) {
                    const float ok = __shfl_xor_sync(0xffffffffu, kk[e], lm);
                    const int ov = __shfl_xor_sync(0xffffffffu, vv[e], lm);
                    const int i = lane * E + e;
                    const bool lower = (i & j) == 0;
                    const bool fwd = (i & ks) == 0;
                    // the lower index keeps the element that sorts first in this block's order
                    const bool mine_first = before(kk[e], vv[e], ok, ov);
                    const bool keep_mine = (lower == fwd) ? mine_first : !mine_first;
                    if (!keep_mine) {
                        kk[e] = ok;
                        vv[e] = ov;
                    }
                }
            }
        }
    }
#pragma unroll
    for (int e = 0; e < E; ++e) {
        const int i = lane * E + e;
        if (i < k) {
            key[i] = kk[e];
            val[i] = vv[e];
        }
    }
}

__device__ int block_topk(const float* key, const int* val, int n, int n_valid, int K, float* okey, int* oval,
                          SelScratch& sc) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int k = min(K, n_valid);
    const bool all = k == n_valid;
    unsigned prefix = 0u, mask = 0u;
    int need = k;  // pairs still to take among those matching prefix
    if (!all) {
        for (int i = tid; i < 512; i += blockDim.x) (&sc.hist[0][0])[i] = 0;
        if (tid == 0) sc.n_out = 0;
        __syncthreads();
        for (int pass = 0; pass < 4; ++pass) {
            const int shift = 24 - 8 * pass;
            int* hist = sc.hist[pass & 1];
            for (int i = tid; i < n; i += blockDim.x) {
                if (val[i] < 0) continue;
                const unsigned u = key_bits(key[i]);
                if ((u & mask) == prefix) atomicAdd(&hist[(u >> shift) & 255u], 1);
            }
            __syncthreads();
            if (warp == 0) {  // digit d: count(digits > d) < need <= count(digits >= d)
                int c[8], sum = 0;
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    c[q] = hist[255 - (lane * 8 + q)];  // lane 0 holds the highest digits
                    sum += c[q];
                }
                int incl = sum;  // inclusive scan over lanes (from the highest digits)
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const int y = __shfl_up_sync(0xffffffffu, incl, o);
                    if (lane >= o) incl += y;
                }
                int run = incl - sum;  // count of digits above this lane's block
                int found = -1, above = 0;
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    if (found < 0 && run + c[q] >= need) {
                        found = 255 - (lane * 8 + q);
                        above = run;
                    }
                    run += c[q];
                }
                const unsigned hit = __ballot_sync(0xffffffffu, found >= 0);
                const int src = __ffs(hit) - 1;
                const int d = __shfl_sync(0xffffffffu, found, src);
                const int ab = __shfl_sync(0xffffffffu, above, src);
                if (lane == 0) {
                    sc.digit = d;
                    sc.above = ab;
                }
            } else {
                // the other buffer (last read by the previous pass's scan) for the next pass
                int* next = sc.hist[(pass + 1) & 1];
                for (int i = tid - 32; i < 256; i += blockDim.x - 32) next[i] = 0;
            }
            __syncthreads();
            prefix |= (unsigned)sc.digit << shift;
            mask |= 255u << shift;
            need -= sc.above;
        }
    } else {
        if (tid == 0) sc.n_out = 0;
        __syncthreads();
    }
    // gather: everything strictly above the threshold (any order), then `need` ties in index order
    for (int i = tid; i < n; i += blockDim.x) {
        if (val[i] < 0) continue;
        if (all || key_bits(key[i]) > prefix) {
            const int slot = atomicAdd(&sc.n_out, 1);
            okey[slot] = key[i];
            oval[slot] = val[i];
        }
    }
    __syncthreads();
    if (!all && need > 0) {
        const int base = sc.n_out;
        int taken = 0;  // ties taken by earlier passes over the array
        for (int i0 = 0; i0 < n && taken < need; i0 += blockDim.x) {
            const int i = i0 + tid;
            const bool tie = i < n && val[i] >= 0 && key_bits(key[i]) == prefix;
            const unsigned bal = __ballot_sync(0xffffffffu, tie);
            if (lane == 0) sc.warp_cnt[warp] = __popc(bal);
            __syncthreads();
            int before_w = 0, total = 0;
            for (int w = 0; w < kBeamThreads / 32; ++w) {
                if (w < warp) before_w += sc.warp_cnt[w];
                total += sc.warp_cnt[w];
            }
            const int rank = taken + before_w + __popc(bal & ((1u << lane) - 1u));
            if (tie && rank < need) {
                okey[base + rank] = key[i];
                oval[base + rank] = val[i];
            }
            taken += total;
            __syncthreads();
        }
    }
    // sort the k winners into `before` order
    if (warp == 0) {
        if (k <= 64)
            warp_sort<2>(okey, oval, k);
        else
            warp_sort<4>(okey, oval, k);
    }
    __syncthreads();
    return k;
}

// Top (K) non-blank tokens of every frame, in `before` order (larger log-prob,
// then lower id), one warp per (utterance, frame) row: each lane holds its
// strided share of the row in registers and K rounds of a warp argmax take the
// next token. Only frames t < in_lens[b] are written. The frames are independent
// of the beam, so this runs over the whole batch in parallel ahead of the search.
constexpr int kTopPerLane = 64;  // vocabularies up to 32 * 64 + 1 columns

__global__ void __launch_bounds__(256) top_tokens_kernel(const float* __restrict__ lp,
                                                         const int32_t* __restrict__ in_lens, int B, int T, int V,
                                                         int K, int32_t* __restrict__ top_tok,
                                                         float* __restrict__ top_lp) {
    const int lane = threadIdx.x & 31;
    const int64_t r = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    if (r >= (int64_t)B * T) return;
    const int b = (int)(r / T), t = (int)(r % T);
    if (t >= min(max(in_lens[b], 0), T)) return;
    const float* row = lp + r * V;
    float x[kTopPerLane];
#pragma unroll
    for (int q = 0; q < kTopPerLane; ++q) {
        const int v = 1 + lane + 32 * q;
        x[q] = v < V ? __ldg(row + v) : -INFINITY;
    }
    unsigned long long taken = 0ull;
    for (int k = 0; k < K; ++k) {
        float bv = -INFINITY;
        int bi = INT_MAX;
#pragma unroll
        for (int q = 0; q < kTopPerLane; ++q) {
            const int v = 1 + lane + 32 * q;
            if (v < V && !((taken >> q) & 1ull) && before(x[q], v, bv, bi)) {
                bv = x[q];
                bi = v;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (before(ov, oi, bv, bi)) {
                bv = ov;
                bi = oi;
            }
        }
        if (((bi - 1) & 31) == lane) taken |= 1ull << ((bi - 1) >> 5);
        if (lane == 0) {
            top_tok[r * K + k] = bi;
            top_lp[r * K + k] = bv;
        }
    }
}

struct Beam {
    int node[kMaxBeam], len[kMaxBeam], last[kMaxBeam];
    float pb[kMaxBeam], pnb[kMaxBeam];
    unsigned long long hash[kMaxBeam];
};

__global__ void __launch_bounds__(kBeamThreads) ctc_beam_kernel(const float* __restrict__ lp,
                                                               const int32_t* __restrict__ in_lens, int T, int V,
                                                               int W, int NT, int NC, int32_t* __restrict__ pool_par,
                                                               int32_t* __restrict__ pool_tok, int64_t pool_cap,
                                                               int32_t* __restrict__ out_tokens,
                                                               int32_t* __restrict__ out_len,
                                                               const int32_t* __restrict__ top_tok,
                                                               const float* __restrict__ top_lp) {
    extern __shared__ __align__(16) unsigned char beam_smem[];
    float* tkey = reinterpret_cast<float*>(beam_smem);  // NT: frame log-probs of tokens 1..V-1
    int* tval = reinterpret_cast<int*>(tkey + NT);
    float* ckey = reinterpret_cast<float*>(tval + NT);  // NC: candidate scores
    int* cval = reinterpret_cast<int*>(ckey + NC);
    unsigned char* mflag = reinterpret_cast<unsigned char*>(cval + NC);  // NC: extension merged into a stay
    __shared__ float skey[kSelMax];  // selected (sorted) top tokens / candidates
    __shared__ int sval[kSelMax];
    __shared__ SelScratch sc;
    __shared__ Beam bs[2];
    __shared__ float spb[kMaxBeam], spnb[kMaxBeam];  // stay candidates (merged)
    __shared__ int toks[kMaxBeam + 1];
    __shared__ float tlp[kMaxBeam + 1];
    __shared__ int s_n, s_cur, s_next, s_valid, s_ext[2];

    const int b = blockIdx.x, tid = threadIdx.x;
    const int Tb = min(max(in_lens[b], 0), T);
    int32_t* par = pool_par + (int64_t)b * pool_cap;
    int32_t* tokp = pool_tok + (int64_t)b * pool_cap;
    if (tid == 0) {
        Beam& c = bs[0];
        c.node[0] = 0;
        c.len[0] = 0;
        c.last[0] = -1;
        c.pb[0] = 0.f;
        c.pnb[0] = -INFINITY;
        c.hash[0] = 0ull;
        par[0] = -1;
        tokp[0] = -1;
        s_n = 1;
        s_cur = 0;
        s_next = 1;
    }
    __syncthreads();
    const int ntop = min(W + 1, V - 1);
    const int per = ntop + 1;  // candidates per entry: the stay, then one per top token

    for (int t = 0; t < Tb; ++t) {
        const float* row = lp + ((int64_t)b * T + t) * V;
        const int cur = s_cur, n = s_n;
        const Beam& c = bs[cur];
        Beam& nx = bs[cur ^ 1];
        // 1. the frame's top non-blank tokens (precomputed for the whole batch when the
        // vocabulary fits the pre-pass, else selected here)
        if (top_tok) {
            if (tid < ntop) {
                const int64_t o = ((int64_t)b * T + t) * ntop + tid;
                toks[tid] = __ldg(top_tok + o);
                tlp[tid] = __ldg(top_lp + o);
            }
        } else {
            for (int i = tid; i < V - 1; i += blockDim.x) {
                tkey[i] = __ldg(row + i + 1);
                tval[i] = i + 1;
            }
            __syncthreads();
            block_topk(tkey, tval, V - 1, V - 1, ntop, skey, sval, sc);
            if (tid < ntop) {
                toks[tid] = sval[tid];
                tlp[tid] = skey[tid];
            }
        }
        __syncthreads();
        // 2. stay candidates, with the parent's extension merged in
        if (tid == 0) s_valid = 0;
        for (int i = tid; i < n * per; i += blockDim.x) mflag[i] = 0;
        __syncthreads();
        if (tid < n) {
            const int e = tid, last = c.last[e];
            float pnb = last >= 0 ? c.pnb[e] + __ldg(row + last) : -INFINITY;
            int pe = -1, pos = -1;
            if (c.len[e] > 0) {
                for (int q = 0; q < n; ++q)
                    if (c.len[q] + 1 == c.len[e] && c.hash[q] * kHashMul + (unsigned long long)(last + 1) == c.hash[e]) {
                        pe = q;
                        break;
                    }
            }
            if (pe >= 0) {
                const float base = last == c.last[pe] ? c.pb[pe] : lae_ref(c.pb[pe], c.pnb[pe]);
                pnb = lae_ref(pnb, base + __ldg(row + last));
                for (int j = 0; j < ntop; ++j)
                    if (toks[j] == last) {
                        pos = j;
                        break;
                    }
            }
            spb[e] = lae_ref(c.pb[e], c.pnb[e]) + __ldg(row);
            spnb[e] = pnb;
            if (pe >= 0 && pos >= 0) mflag[pe * per + 1 + pos] = 1;  // that extension is this stay
        }
        __syncthreads();
        // 3. candidate scores (s_valid counts the candidates that stay)
        const int nc = n * per;
        for (int i = tid; i < nc; i += blockDim.x) {
            float key = -INFINITY;
            int val = -1;
            if (i < nc) {
                const int e = i / per, j = i - e * per;
                if (j == 0) {
                    key = lae_ref(spb[e], spnb[e]);
                    val = i;
                } else {
                    if (!mflag[i]) {
                        const int v = toks[j - 1];
                        const float base = v == c.last[e] ? c.pb[e] : lae_ref(c.pb[e], c.pnb[e]);
                        key = base + tlp[j - 1];
                        val = i;
                    }
                }
            }
            ckey[i] = key;
            cval[i] = val;
            if (val >= 0) atomicAdd(&s_valid, 1);
        }
        __syncthreads();
        const int keep = block_topk(ckey, cval, nc, s_valid, W, skey, sval, sc);
        // 4. the next beam (W entries at most): thread k builds entry k; new prefixes
        // get pool nodes numbered in entry order (a ballot scan over warps 0-1)
        {
            const bool mine = tid < keep;
            const int i = mine ? sval[tid] : 0, e = i / per, j = i - e * per;
            const bool ext = mine && j != 0;
            const unsigned bal = __ballot_sync(0xffffffffu, ext);
            if (lane_of(tid) == 0 && tid < 64) s_ext[tid >> 5] = __popc(bal);
            __syncthreads();
            if (mine) {
                if (!ext) {
                    nx.node[tid] = c.node[e];
                    nx.len[tid] = c.len[e];
                    nx.last[tid] = c.last[e];
                    nx.pb[tid] = spb[e];
                    nx.pnb[tid] = spnb[e];
                    nx.hash[tid] = c.hash[e];
                } else {
                    const int rank = (tid >= 32 ? s_ext[0] : 0) + __popc(bal & ((1u << (tid & 31)) - 1u));
                    const int node = s_next + rank;
                    const int v = toks[j - 1];
                    par[node] = c.node[e];
                    tokp[node] = v;
                    nx.node[tid] = node;
                    nx.len[tid] = c.len[e] + 1;
                    nx.last[tid] = v;
                    nx.pb[tid] = -INFINITY;
                    nx.pnb[tid] = skey[tid];
                    nx.hash[tid] = c.hash[e] * kHashMul + (unsigned long long)(v + 1);
                }
            }
            __syncthreads();
            if (tid == 0) {
                s_n = keep;
                s_next += s_ext[0] + (keep > 32 ? s_ext[1] : 0);
                s_cur = cur ^ 1;
            }
            __syncthreads();
        }
    }
    // 5. the best surviving prefix, backtracked through the node pool
    if (tid == 0) {
        const Beam& c = bs[s_cur];
        int best = 0;
        float bt = lae_ref(c.pb[0], c.pnb[0]);
        for (int e = 1; e < s_n; ++e) {
            const float x = lae_ref(c.pb[e], c.pnb[e]);
            if (x > bt) {
                bt = x;
                best = e;
            }
        }
        const int L = c.len[best];
        int node = c.node[best];
        out_len[b] = L;
        for (int i = L - 1; i >= 0; --i) {
            out_tokens[(int64_t)b * T + i] = tokp[node];
            node = par[node];
        }
    }
}

}  // namespace
}  // namespace asr

using namespace asr;

extern "C" size_t asr_ctc_beam_workspace_bytes(int B, int T, int beam_width) {
    if (B < 0 || T < 0 || beam_width < 1 || beam_width > kMaxBeam) return 0;
    // node pool (parent, token) + the per-frame top-token table (id, log-prob)
    return sizeof(int32_t) * 2 * (size_t)B * (1 + (size_t)T * beam_width) +
           sizeof(int32_t) * 2 * (size_t)B * T * (beam_width + 1) + 512;
}

extern "C" int asr_ctc_beam_decode(const float* log_probs, const int32_t* in_lens, int B, int T, int V,
                                   int beam_width, int32_t* tokens, int32_t* lengths, void* workspace,
                                   size_t workspace_bytes, asr_stream_t stream) {
    if (B < 0 || T < 0 || V < 1 || beam_width < 1) return ASR_ERR_INVALID_ARGUMENT;
    if (B == 0) return ASR_OK;
    if (!log_probs || !in_lens || !tokens || !lengths) return ASR_ERR_INVALID_ARGUMENT;
    if (beam_width > kMaxBeam || V > kMaxBeamVocab) return ASR_ERR_UNSUPPORTED;
    if (!workspace || workspace_bytes < asr_ctc_beam_workspace_bytes(B, T, beam_width)) return ASR_ERR_WORKSPACE;
    const int ntop = std::min(beam_width + 1, V - 1);
    const int NT = std::max(V - 1, 1);
    const int NC = beam_width * (ntop + 1);
    const int64_t cap = 1 + (int64_t)T * beam_width;
    auto* base = reinterpret_cast<int32_t*>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255));
    const size_t smem = sizeof(float) * 2 * (size_t)(NT + NC) + (size_t)NC;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (smem > 48 * 1024)
        ASR_CUDA_TRY(cudaFuncSetAttribute(ctc_beam_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    if (T == 0) {
        ASR_CUDA_TRY(cudaMemsetAsync(lengths, 0, sizeof(int32_t) * B, st));
        return ASR_OK;
    }
    int32_t* top_tok = nullptr;
    float* top_lp = nullptr;
    if (V - 1 <= 32 * kTopPerLane && ntop > 0) {
        int32_t* tbl = base + 2 * (size_t)B * cap;
        top_tok = tbl;
        top_lp = reinterpret_cast<float*>(tbl + (size_t)B * T * ntop);
        KernelTimer kt("ctc_beam_top_tokens", st);
        const int64_t rows = (int64_t)B * T;
        top_tokens_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(log_probs, in_lens, B, T, V, ntop, top_tok,
                                                                      top_lp);
        ASR_LAUNCH_CHECK();
    }
    KernelTimer kt("ctc_beam", st);
    ctc_beam_kernel<<<B, kBeamThreads, smem, st>>>(log_probs, in_lens, T, V, beam_width, NT, NC, base,
                                                   base + (size_t)B * cap, cap, tokens, lengths, top_tok, top_lp);
    ASR_LAUNCH_CHECK();
    return ASR_OK;
}
