// fp32-accurate joint network (SIMT FMA), the tf32 = 0 mode of the reference.
//
// Forward: one kernel per 64-node tile. The hidden tile tanh(enc + dec) is
// built on the fly into shared memory, multiplied against 64-column slices of
// the full output projection [joint_W; joint_W_dur], and each slice is folded
// into a per-node online log-sum-exp while the blank / label / duration logits
// are gathered. Only five floats per node (plus the duration log-probs) reach
// HBM; the logits never do.
// Backward, per chunk of nodes: (1) recompute the logits and turn them into
// d loss / d logits with the saved log-partition and the beta-pass posteriors
// (G, fp32 scratch); (2) dH = G * Wf with tanh' applied in the epilogue and
// scattered to d_enc / d_dec; (3) dW = G^T * hidden as a split-K GEMM whose B
// operand (hidden) is recomputed on the fly.
#include <algorithm>
#include <cfloat>

#include "joint.cuh"

namespace asr {
namespace {

constexpr int BM = 64, BN = 64, BK = 16, NT = 256;
constexpr int kMaxDur = 32;

__device__ __forceinline__ float wfull(const JointArgs& a, int c, int k) {
    if (c < a.V) return __ldg(a.W + (int64_t)c * a.d + k);
    c -= a.V;
    if (c < a.n_dur) return __ldg(a.Wd + (int64_t)c * a.d + k);
    return 0.f;
}

// 64x64 register-blocked tile product over one BK slice held in shared memory.
__device__ __forceinline__ void mma_slice(const float (&As)[BK][BM + 4], const float (&Bs)[BK][BN + 4],
                                          float (&acc)[4][4], int ty, int tx) {
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
        float av[4], bv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) av[i] = As[kk][ty + 16 * i];
#pragma unroll
        for (int j = 0; j < 4; ++j) bv[j] = Bs[kk][tx + 16 * j];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
}

struct RowInfo {
    int64_t enc, dec;  // element offsets of the encoder / decoder rows
    int y;             // emitted label, -1 without a label edge
    int n;             // compact node id, -1 for an empty tile row
    int dn;            // its place in the utterance's diagonal-major weight block
};

__device__ __forceinline__ RowInfo make_row(const JointArgs& a, int n, int N) {
    RowInfo r;
    if (n < 0 || n >= N) {
        r.enc = r.dec = 0;
        r.y = -1;
        r.n = -1;
        r.dn = -1;
        return r;
    }
    const NodeCoord c = node_coord(a.m, a.B, n);
    r.enc = ((int64_t)c.b * a.T + c.t) * a.d;
    r.dec = ((int64_t)c.b * a.U + c.u) * a.d;
    r.y = (c.u < c.Ub - 1) ? __ldg(a.targets + (int64_t)c.b * a.S + c.u) : -1;
    r.n = n;
    r.dn = __ldg(a.m.off + c.b) + diag_index(c.t, c.u, __ldg(a.m.Tb + c.b), c.Ub);
    return r;
}

// Loads the hidden slice As[kk][r] = tanh(enc + dec) for the tile rows.
__device__ __forceinline__ void load_hidden(const JointArgs& a, const RowInfo* rows, int kc, float (&As)[BK][BM + 4],
                                            int tid) {
#pragma unroll
    for (int q = 0; q < (BM * BK) / NT; ++q) {
        const int e = tid + NT * q;
        const int r = e / BK, kk = e % BK;
        float h = 0.f;
        if (rows[r].n >= 0 && kc + kk < a.d)
            h = tanhf(__ldg(a.enc + rows[r].enc + kc + kk) + __ldg(a.dec + rows[r].dec + kc + kk));
        As[kk][r] = h;
    }
}

__device__ __forceinline__ void load_wslice(const JointArgs& a, int vc, int kc, float (&Bs)[BK][BN + 4], int tid) {
    const int Vf = a.V + a.n_dur;
#pragma unroll
    for (int q = 0; q < (BN * BK) / NT; ++q) {
        const int e = tid + NT * q;
        const int c = e / BK, kk = e % BK;
        Bs[kk][c] = (vc + c < Vf && kc + kk < a.d) ? wfull(a, vc + c, kc + kk) : 0.f;
    }
}

__global__ void __launch_bounds__(NT) simt_fwd_kernel(JointArgs a, JointFwdOut o) {
    __shared__ float As[BK][BM + 4], Bs[BK][BN + 4];
    __shared__ float Ls[BM][BN + 1];
    __shared__ RowInfo rows[BM];
    __shared__ float r_m[BM], r_s[BM], r_blank[BM], r_lab[BM];
    __shared__ float r_dur[BM][kMaxDur];
    const int tid = threadIdx.x, tx = tid % 16, ty = tid / 16;
    const int N = total_nodes(a.m, a.B);
    const int Vf = a.V + a.n_dur;
    const int ntiles = (N + BM - 1) / BM;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
        if (tid < BM) {
            rows[tid] = make_row(a, tile * BM + tid, N);
            r_m[tid] = -INFINITY;
            r_s[tid] = 0.f;
            r_blank[tid] = 0.f;
            r_lab[tid] = 0.f;
        }
        __syncthreads();
        for (int vc = 0; vc < Vf; vc += BN) {
            float acc[4][4] = {};
            for (int kc = 0; kc < a.d; kc += BK) {
                load_hidden(a, rows, kc, As, tid);
                load_wslice(a, vc, kc, Bs, tid);
                __syncthreads();
                mma_slice(As, Bs, acc, ty, tx);
                __syncthreads();
            }
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) Ls[ty + 16 * i][tx + 16 * j] = acc[i][j];
            __syncthreads();
            // online log-sum-exp over the token columns of this slice; 4 lanes per row
            {
                const int row = tid >> 2, part = tid & 3;
                const RowInfo& ri = rows[row];
                float mx = -INFINITY;
                for (int c = part * 16; c < part * 16 + 16; ++c) {
                    const int v = vc + c;
                    if (v < a.V) mx = fmaxf(mx, Ls[row][c]);
                }
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
                const float m_old = r_m[row];
                const float m_new = fmaxf(m_old, mx);
                float s = 0.f;
                for (int c = part * 16; c < part * 16 + 16; ++c) {
                    const int v = vc + c;
                    if (v < a.V) s += __expf(Ls[row][c] - m_new);
                }
                s += __shfl_xor_sync(0xffffffffu, s, 1);
                s += __shfl_xor_sync(0xffffffffu, s, 2);
                for (int c = part * 16; c < part * 16 + 16; ++c) {
                    const int v = vc + c;
                    if (v == a.blank) r_blank[row] = Ls[row][c];
                    if (v == ri.y) r_lab[row] = Ls[row][c];
                    if (v >= a.V && v < Vf) r_dur[row][v - a.V] = Ls[row][c];
                }
                if (part == 0 && m_new > -INFINITY) {
                    r_s[row] = (m_old > -INFINITY ? r_s[row] * __expf(m_old - m_new) : 0.f) + s;
                    r_m[row] = m_new;
                }
            }
            __syncthreads();
        }
        if (tid < BM && rows[tid].n >= 0) {
            const int n = rows[tid].n, dn = rows[tid].dn;
            const float lse = r_m[tid] + __logf(r_s[tid]);
            o.lse[n] = lse;
            o.lpb[dn] = r_blank[tid] - lse - a.sigma;
            o.lpy[dn] = rows[tid].y >= 0 ? r_lab[tid] - lse - a.sigma : kNeg;
            if (a.n_dur > 0) {
                float md = -INFINITY;
                for (int k = 0; k < a.n_dur; ++k) md = fmaxf(md, r_dur[tid][k]);
                float sd = 0.f;
                for (int k = 0; k < a.n_dur; ++k) sd += __expf(r_dur[tid][k] - md);
                const float lz = md + __logf(sd);
                for (int k = 0; k < a.n_dur; ++k) o.lpd[(int64_t)dn * a.n_dur + k] = r_dur[tid][k] - lz;
            }
        }
        __syncthreads();
    }
}

// G[n - c0, c] = d loss / d logits for the nodes of chunk [c0, c0 + cn).
__global__ void __launch_bounds__(NT) simt_bwd_g_kernel(JointArgs a, JointBwdIn in, float* __restrict__ G, int c0,
                                                        int cn) {
    __shared__ float As[BK][BM + 4], Bs[BK][BN + 4];
    __shared__ RowInfo rows[BM];
    __shared__ float r_lse[BM], r_cb[BM], r_ct[BM];
    const int tid = threadIdx.x, tx = tid % 16, ty = tid / 16;
    const int N = total_nodes(a.m, a.B);
    const int end = min(N, c0 + cn);
    const int Vf = a.V + a.n_dur;
    const int vtiles = (Vf + BN - 1) / BN;
    const int ntiles = (max(end - c0, 0) + BM - 1) / BM;
    for (int w = blockIdx.x; w < ntiles * vtiles; w += gridDim.x) {
        const int tile = w / vtiles, vc = (w % vtiles) * BN;
        if (tid < BM) {
            const int n = c0 + tile * BM + tid;
            rows[tid] = make_row(a, n < end ? n : -1, N);
            if (rows[tid].n >= 0) {
                r_lse[tid] = in.lse[n];
                r_cb[tid] = in.cb[n];
                r_ct[tid] = in.ct[n];
            }
        }
        __syncthreads();
        float acc[4][4] = {};
        for (int kc = 0; kc < a.d; kc += BK) {
            load_hidden(a, rows, kc, As, tid);
            load_wslice(a, vc, kc, Bs, tid);
            __syncthreads();
            mma_slice(As, Bs, acc, ty, tx);
            __syncthreads();
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int r = ty + 16 * i;
            const RowInfo ri = rows[r];
            if (ri.n < 0) continue;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int v = vc + tx + 16 * j;
                if (v >= Vf) continue;
                float g;
                if (v < a.V) {
                    g = __expf(acc[i][j] - r_lse[r]) * (r_cb[r] + r_ct[r]);
                    if (v == a.blank) g -= r_cb[r];
                    if (v == ri.y) g -= r_ct[r];
                } else {
                    g = in.gdur[(int64_t)ri.n * a.n_dur + (v - a.V)];
                }
                G[(int64_t)(ri.n - c0) * Vf + v] = g;
            }
        }
        __syncthreads();
    }
}

// d_enc / d_dec += (G * Wf) * (1 - hidden^2), summed over the other lattice axis.
__global__ void __launch_bounds__(NT) simt_dh_kernel(JointArgs a, const float* __restrict__ G, JointBwdOut o, int c0,
                                                     int cn) {
    __shared__ float As[BK][BM + 4], Bs[BK][BN + 4];
    __shared__ RowInfo rows[BM];
    const int tid = threadIdx.x, tx = tid % 16, ty = tid / 16;
    const int N = total_nodes(a.m, a.B);
    const int end = min(N, c0 + cn);
    const int Vf = a.V + a.n_dur;
    const int dtiles = (a.d + BN - 1) / BN;
    const int ntiles = (max(end - c0, 0) + BM - 1) / BM;
    for (int w = blockIdx.x; w < ntiles * dtiles; w += gridDim.x) {
        const int tile = w / dtiles, dc = (w % dtiles) * BN;
        if (tid < BM) {
            const int n = c0 + tile * BM + tid;
            rows[tid] = make_row(a, n < end ? n : -1, N);
        }
        __syncthreads();
        float acc[4][4] = {};
        for (int kc = 0; kc < Vf; kc += BK) {
#pragma unroll
            for (int q = 0; q < (BM * BK) / NT; ++q) {
                const int e = tid + NT * q;
                const int r = e / BK, kk = e % BK;
                As[kk][r] = (rows[r].n >= 0 && kc + kk < Vf) ? G[(int64_t)(rows[r].n - c0) * Vf + kc + kk] : 0.f;
            }
#pragma unroll
            for (int q = 0; q < (BN * BK) / NT; ++q) {
                const int e = tid + NT * q;
                const int c = e % BN, kk = e / BN;
                Bs[kk][c] = (kc + kk < Vf && dc + c < a.d) ? wfull(a, kc + kk, dc + c) : 0.f;
            }
            __syncthreads();
            mma_slice(As, Bs, acc, ty, tx);
            __syncthreads();
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const RowInfo ri = rows[ty + 16 * i];
            if (ri.n < 0) continue;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int k = dc + tx + 16 * j;
                if (k >= a.d) continue;
                const float h = tanhf(__ldg(a.enc + ri.enc + k) + __ldg(a.dec + ri.dec + k));
                const float gp = acc[i][j] * (1.f - h * h);
                atomicAdd(o.d_enc + ri.enc + k, gp);
                atomicAdd(o.d_dec + ri.dec + k, gp);
            }
        }
        __syncthreads();
    }
}

// dW[c, k] += sum_n G[n, c] * hidden[n, k] over a split of the chunk's nodes.
__global__ void __launch_bounds__(NT) simt_dw_kernel(JointArgs a, const float* __restrict__ G, JointBwdOut o, int c0,
                                                     int cn, int per_split) {
    __shared__ float As[BK][BM + 4], Bs[BK][BN + 4];
    __shared__ RowInfo krow[BK];
    const int tid = threadIdx.x, tx = tid % 16, ty = tid / 16;
    const int N = total_nodes(a.m, a.B);
    const int end = min(N, c0 + cn);
    const int Vf = a.V + a.n_dur;
    const int vc = blockIdx.x * BM, dc = blockIdx.y * BN;
    const int s0 = c0 + blockIdx.z * per_split;
    const int s1 = min(end, s0 + per_split);
    if (s0 >= s1) return;
    float acc[4][4] = {};
    for (int nb = s0; nb < s1; nb += BK) {
        if (tid < BK) krow[tid] = make_row(a, nb + tid < s1 ? nb + tid : -1, N);
        __syncthreads();
#pragma unroll
        for (int q = 0; q < (BM * BK) / NT; ++q) {
            const int e = tid + NT * q;
            const int r = e % BM, kk = e / BM;
            As[kk][r] = (krow[kk].n >= 0 && vc + r < Vf) ? G[(int64_t)(krow[kk].n - c0) * Vf + vc + r] : 0.f;
        }
#pragma unroll
        for (int q = 0; q < (BN * BK) / NT; ++q) {
            const int e = tid + NT * q;
            const int c = e % BN, kk = e / BN;
            float h = 0.f;
            if (krow[kk].n >= 0 && dc + c < a.d)
                h = tanhf(__ldg(a.enc + krow[kk].enc + dc + c) + __ldg(a.dec + krow[kk].dec + dc + c));
            Bs[kk][c] = h;
        }
        __syncthreads();
        mma_slice(As, Bs, acc, ty, tx);
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int v = vc + ty + 16 * i;
        if (v >= Vf) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int k = dc + tx + 16 * j;
            if (k >= a.d) continue;
            if (v < a.V)
                atomicAdd(o.dW + (int64_t)v * a.d + k, acc[i][j]);
            else
                atomicAdd(o.dWd + (int64_t)(v - a.V) * a.d + k, acc[i][j]);
        }
    }
}

constexpr int kSimtChunk = 65536;

}  // namespace

int simt_joint_forward(const JointArgs& a, const JointFwdOut& o, cudaStream_t st) {
    if (a.n_dur > kMaxDur) return ASR_ERR_UNSUPPORTED;
    const int cap_tiles = (int)(((int64_t)a.B * a.T * a.U + BM - 1) / BM);
    const int grid = std::max(1, std::min(cap_tiles, sm_count() * 6));
    {
        KernelTimer kt("joint_fwd_simt", st);
        simt_fwd_kernel<<<grid, NT, 0, st>>>(a, o);
    }
    ASR_LAUNCH_CHECK();
    return ASR_OK;
}

size_t simt_backward_scratch_bytes(int Vf, int chunk) { return sizeof(float) * (size_t)Vf * std::min(chunk, kSimtChunk); }

int simt_joint_backward(const JointArgs& a, const JointBwdIn& in, const JointBwdOut& o, int node_capacity,
                        void* scratch, size_t scratch_bytes, cudaStream_t st) {
    const int Vf = a.V + a.n_dur;
    const int chunk = std::min(node_capacity, kSimtChunk);
    if (scratch_bytes < sizeof(float) * (size_t)Vf * chunk) return ASR_ERR_WORKSPACE;
    float* G = static_cast<float*>(scratch);
    const int sms = sm_count();
    for (int c0 = 0; c0 < node_capacity; c0 += chunk) {
        const int cn = std::min(chunk, node_capacity - c0);
        const int ntiles = (cn + BM - 1) / BM;
        const int vt = (Vf + BN - 1) / BN, dt = (a.d + BN - 1) / BN;
        {
            KernelTimer kt("joint_dlogits_simt", st);
            simt_bwd_g_kernel<<<std::max(1, std::min(ntiles * vt, sms * 6)), NT, 0, st>>>(a, in, G, c0, cn);
        }
        ASR_LAUNCH_CHECK();
        {
            KernelTimer kt("joint_dhidden_simt", st);
            simt_dh_kernel<<<std::max(1, std::min(ntiles * dt, sms * 6)), NT, 0, st>>>(a, G, o, c0, cn);
        }
        ASR_LAUNCH_CHECK();
        const int out_tiles = ((Vf + BM - 1) / BM) * dt;
        const int splits = std::max(1, std::min((sms * 4 + out_tiles - 1) / out_tiles, (cn + 255) / 256));
        const int per = (((cn + splits - 1) / splits) + BK - 1) / BK * BK;
        dim3 g((Vf + BM - 1) / BM, dt, splits);
        {
            KernelTimer kt("joint_dweight_simt", st);
            simt_dw_kernel<<<g, NT, 0, st>>>(a, G, o, c0, cn, per);
        }
        ASR_LAUNCH_CHECK();
    }
    return ASR_OK;
}

}  // namespace asr
