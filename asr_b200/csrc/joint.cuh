// Joint network + fused epilogues: shared argument block and launchers for the
// fp32 SIMT path (joint_simt.cu) and the bf16 tcgen05 path (joint_tc.cu).
//
// The joint output is  logits[n, c] = sum_k tanh(enc[b,t,k] + dec[b,u,k]) * Wf[c, k]
// over the compact valid nodes n = (b, t, u) and the "full" column set
// c in [0, Vf), Vf = V + n_dur: token columns first (joint_W), then the duration
// head (joint_W_dur). The fp32 logits never reach HBM; the tensor-core forward
// can keep a reduced-width copy for the backward (LogitStash).
#pragma once

#include <cuda_bf16.h>

#include "common.cuh"

namespace asr {

struct JointArgs {
    const float* enc;      // (B, T, d) fp32 activations, or nullptr when enc16 is set
    const float* dec;      // (B, U, d)
    const __nv_bfloat16* enc16;  // bf16 activations (the tensor-core path reads them directly)
    const __nv_bfloat16* dec16;
    int vec;               // d % 8 == 0 and 16-byte aligned activation bases: vector row loads
    const float* W;        // (V, d)
    const float* Wd;       // (n_dur, d) or nullptr
    const int32_t* targets;  // (B, S)
    LatticeMeta m;
    int B, T, U, V, n_dur, d, S, blank;
    float sigma;
    // CTC head mode (head = 1, tensor-core path only): the lattice has one label
    // position per frame (U_b = 1) and the hidden row is RMSNorm(enc) * rms_g
    // instead of tanh(enc + dec); with `bias` the GEMM gains a ones column whose
    // weight column is the bias (K = d + 1). dec / targets are unused.
    int head;
    const float* rms_g;  // (d,) RMSNorm weight
    float rms_eps;
    const float* bias;   // (V,) or nullptr
    // Tensor-core path only. 0: bf16 operands (tf32 = 1). 1: fp32 accuracy from
    // three bf16 products (tf32 = 0): each fp32 operand x = hi + lo with hi =
    // bf16(x), lo = bf16(x - hi), and every GEMM sums hi*hi + lo*hi + hi*lo in
    // fp32 (the dropped lo*lo and the rounding of lo are ~2^-16 of the product).
    int split;
};

// Forward epilogue outputs (compact per-node arrays). The lattice weights the
// recursions read (lpb, lpy, lpd) are stored diagonal-major within each
// utterance's block (diag_index over its T_b x U_b grid); lse, read back by the
// backward joint, is node-major.
struct JointFwdOut {
    float* lpb;  // blank log-prob (minus sigma), diagonal-major
    float* lse;  // token log-partition, node-major
    float* lpy;  // label log-prob (minus sigma), kNeg without a label edge, diagonal-major
    float* lpd;  // (nodes, n_dur) duration log-probs, diagonal-major, or nullptr
};

// Backward: per-node coefficients from the beta pass and the gradient outputs.
struct JointBwdIn {
    const float* lse;   // token log-partition (forward)
    const float* cb;    // grad_loss * blank posterior
    const float* ct;    // grad_loss * label posterior
    const float* gdur;  // (nodes, n_dur) d loss / d duration logit, or nullptr
};

struct JointBwdOut {
    float* d_enc;  // (B, T, d), accumulated (CTC head mode: d loss / d hidden row, before RMSNorm)
    float* d_dec;  // (B, U, d), accumulated (unused in CTC head mode)
    float* dW;     // (V, d), accumulated
    float* dWd;    // (n_dur, d), accumulated, or nullptr
    float* dbias;  // (V,), accumulated: CTC head mode with a bias, else nullptr
};

// Logit stash (tensor-core path): the forward keeps the logits of the first
// `nodes` compact lattice nodes, and the backward forms their rows of
// d loss / d logits in one streaming pass over the stash instead of recomputing
// the logits GEMM; nodes past the stash are recomputed as before. Row n holds
// x[n, c] = logit[n, c] - ref[n, j] for its vpad columns, ref[n, j] the row's
// largest token logit within vocabulary chunk j (so the entries that carry the
// softmax mass sit near 0): fp16 in the bf16 mode, fp32 in the split fp32 mode.
// Its meta row holds ref[n, 0 .. nchunks), the log-partition lse[n] and the
// label (int bits, -1 without a label edge): what the backward needs of the
// node besides its edge posteriors, in one contiguous run.
struct LogitStash {
    void* data;   // (nodes, vpad) fp16 or fp32
    float* meta;  // (nodes, nchunks + 2)
    int nodes;    // a multiple of 256 (whole tiles of every kernel); 0 = no stash
};
// Bytes of one stashed node; the stash of `bytes` holds
// floor((bytes - 512) / per node) nodes, rounded down to a multiple of 256.
size_t tc_stash_bytes_per_node(const JointArgs& a);
LogitStash tc_stash_carve(const JointArgs& a, void* stash, size_t bytes);

// ---- fp32 SIMT path -----------------------------------------------------------
int simt_joint_forward(const JointArgs& a, const JointFwdOut& o, cudaStream_t st);
// Backward over node chunks [c0, c0 + chunk); G is a (chunk, Vf) fp32 scratch.
size_t simt_backward_scratch_bytes(int Vf, int chunk);
int simt_joint_backward(const JointArgs& a, const JointBwdIn& in, const JointBwdOut& o, int node_capacity,
                        void* scratch, size_t scratch_bytes, cudaStream_t st);

// ---- bf16 tcgen05 path --------------------------------------------------------
bool tc_supported(const JointArgs& a);
size_t tc_forward_scratch_bytes(const JointArgs& a, int node_capacity);
int tc_joint_forward(const JointArgs& a, const JointFwdOut& o, int node_capacity, void* scratch, size_t scratch_bytes,
                     cudaStream_t st, const LogitStash& stash = LogitStash{});
bool tc_backward_supported(const JointArgs& a);
size_t tc_backward_scratch_bytes(const JointArgs& a, int node_capacity);
int tc_joint_backward(const JointArgs& a, const JointBwdIn& in, const JointBwdOut& o, int node_capacity,
                      void* scratch, size_t scratch_bytes, cudaStream_t st, const LogitStash& stash = LogitStash{});

}  // namespace asr
