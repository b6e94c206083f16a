/*
 * asr_b200 — C ABI of the B200 (sm_100a) fused sequence-loss library:
 * CTC, RNN-T and TDT losses with their joint network, forward and backward.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream, is
 * asynchronous on that stream, performs no host<->device synchronisation and
 * allocates no memory: scratch space is passed in as `workspace` (size from the
 * matching *_workspace_bytes query). Inputs are row-major and contiguous, as in
 * the reference ops (src/asr/loss/csrc/rnnt.cu:13-26). A non-zero return is an
 * asr_status_t; kernels are not launched in that case.
 *
 * Lengths follow the reference contract: in_lens[b] in [1, T], tgt_lens[b] in
 * [0, U-1] (and <= S). Out-of-range lengths are clamped into range on the
 * device so no access leaves the buffers (the reference leaves this undefined).
 *
 * Lattice buffers exchanged between forward and backward ("opaque" outputs of
 * the reference ops) hold only the valid nodes of each utterance, packed
 * utterance after utterance with node (t, u) of utterance b at
 * off[b] + t * U_b + u, U_b = tgt_lens[b] + 1; their capacities are the
 * reference tensor sizes, so callers allocate exactly what the reference did,
 * except log_P_blank which carries a second plane (the per-node token
 * log-partition, reused by the backward softmax).
 */
#ifndef ASR_B200_H_
#define ASR_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same object as cudaStream_t; NULL selects the legacy default stream. */
typedef struct CUstream_st* asr_stream_t;

typedef enum {
    ASR_OK = 0,
    ASR_ERR_INVALID_ARGUMENT = 1, /* a size/flag/pointer check failed on the host */
    ASR_ERR_WORKSPACE = 2,        /* workspace missing or smaller than *_workspace_bytes */
    ASR_ERR_UNSUPPORTED = 3,      /* shape outside the compiled kernel range (e.g. U > 8192) */
    ASR_ERR_CUDA = 4,             /* a CUDA launch or runtime call failed */
    ASR_ERR_SCRATCH_LIMIT = 5     /* problem needs more than the fixed scratch of a *_noalloc entry point */
} asr_status_t;

/* Element type of the encoder / decoder activations and of their gradients in
 * the *_ex entry points (the joint weights and every other array stay float32). */
typedef enum {
    ASR_DTYPE_F32 = 0,
    ASR_DTYPE_BF16 = 1
} asr_dtype_t;

/* Human-readable name of a status code. */
const char* asr_status_string(int status);

/* ABI revision of this header (bumped on any signature change). */
int asr_abi_version(void);

/* ------------------------------------------------------------------ CTC */

/* Replaces ctc_alpha_cuda (reference src/asr/loss/csrc/ctc.cu:214-238; op schema
 * asr::ctc_alpha, ctc_bindings.cpp:17).
 * log_probs (B,T,V) log-softmax over V, blank = 0; targets (B,S).
 * Writes alpha (B,T,2S+1), float64, for t < in_lens[b] and log_Z (B,) (-inf when infeasible). */
int asr_ctc_alpha(const float* log_probs, const int32_t* targets, const int32_t* in_lens, const int32_t* tgt_lens,
                  int B, int T, int V, int S, double* alpha, float* log_Z, asr_stream_t stream);

/* Replaces ctc_grad_cuda (ctc.cu:241-269; asr::ctc_grad, ctc_bindings.cpp:19-21).
 * Writes all of grad_logits (B,T,V): d loss_b / d logits for log_probs =
 * log_softmax(logits), scaled by grad_loss[b]; zero rows past in_lens[b] and,
 * with zero_infinity, for utterances whose log Z is not finite. log Z is recomputed in
 * float64 from alpha; the log_Z argument is accepted for interface parity only. */
int asr_ctc_grad(const double* alpha, const float* log_Z, const float* log_probs, const int32_t* targets,
                 const int32_t* in_lens, const int32_t* tgt_lens, const float* grad_loss, int zero_infinity, int B,
                 int T, int V, int S, float* grad_logits, asr_stream_t stream);

/* ---------------------------------------------------------------- RNN-T */

/* Workspace for asr_rnnt_forward (backward = 0) or asr_rnnt_backward (backward = 1). */
size_t asr_rnnt_workspace_bytes(int B, int T, int U, int V, int d, int tf32, int backward);

/* Replaces rnnt_forward_cuda (rnnt.cu:320-380; asr::rnnt_forward, rnnt_bindings.cpp:24-26).
 * encoder (B,T,d), decoder (B,U,d), joint_W (V,d), targets (B,S) with S >= U-1.
 * tf32 = 0: fp32-accurate joint GEMMs (tcgen05 tensor cores on split bf16 operands,
 * three products per fp32 product; fp32 FMA for shapes outside them, see
 * asr_joint_path). tf32 != 0: bf16 tcgen05 tensor-core joint with fp32
 * accumulation (the reference's opt-in fast mode).
 * Outputs: loss (B,) = -log P(y|x); log_prob (B,) = log P(y|x);
 *   alpha        capacity B*T*U      float64 forward variable per valid node;
 *   log_P_blank  capacity 2*B*T*U    plane 0: blank log-prob, plane 1: token log-partition;
 *   log_P_y      capacity B*T*U      label log-prob (-1e30 where no label edge). */
int asr_rnnt_forward(const float* encoder, const float* decoder, const float* joint_W, const int32_t* targets,
                     const int32_t* in_lens, const int32_t* tgt_lens, int B, int T, int U, int V, int d, int S,
                     int blank_idx, int tf32, float* loss, double* alpha, float* log_P_blank, float* log_P_y,
                     float* log_prob, void* workspace, size_t workspace_bytes, asr_stream_t stream);

/* Replaces rnnt_backward_cuda (rnnt.cu:382-458; asr::rnnt_backward, rnnt_bindings.cpp:27-29).
 * Consumes the forward's lattice buffers; writes (overwrites) grad_encoder (B,T,d),
 * grad_decoder (B,U,d), grad_joint_W (V,d), scaled per utterance by grad_loss (B,).
 * log P(y|x) is recomputed in float64 from alpha; log_prob is accepted for
 * interface parity only. */
int asr_rnnt_backward(const float* encoder, const float* decoder, const float* joint_W, const int32_t* targets,
                      const int32_t* in_lens, const int32_t* tgt_lens, int B, int T, int U, int V, int d, int S,
                      int blank_idx, const double* alpha, const float* log_P_blank, const float* log_P_y,
                      const float* log_prob, const float* grad_loss, int tf32, float* grad_encoder,
                      float* grad_decoder, float* grad_joint_W, void* workspace, size_t workspace_bytes,
                      asr_stream_t stream);

/* ------------------------------------------------------------------ TDT */

/* Workspace for asr_tdt_forward (backward = 0) or asr_tdt_backward (backward = 1). */
size_t asr_tdt_workspace_bytes(int B, int T, int U, int V, int n_dur, int d, int tf32, int backward);

/* Replaces tdt_forward_cuda (tdt.cu:523-600; asr::tdt_forward, tdt_bindings.cpp:28-31).
 * joint_W_dur (n_dur,d); durations (n_dur,) device int32, non-negative, containing 1;
 * max_duration = max(durations) (<= 16 supported); has_zero = (0 in durations);
 * sigma >= 0 is subtracted from the blank and label log-probs (tdt.cu:164-165).
 * loss = -alpha[in_lens, tgt_lens] (exact landing).
 * Outputs: alpha capacity B*(T+1)*U (float64); log_P_blank capacity 2*B*T*U (as RNN-T);
 *   log_P_y capacity B*T*U; log_P_dur capacity B*T*U*n_dur. */
int asr_tdt_forward(const float* encoder, const float* decoder, const float* joint_W, const float* joint_W_dur,
                    const int32_t* targets, const int32_t* in_lens, const int32_t* tgt_lens,
                    const int32_t* durations, int n_dur, int max_duration, int has_zero, int B, int T, int U, int V,
                    int d, int S, int blank_idx, float sigma, int tf32, float* loss, double* alpha,
                    float* log_P_blank, float* log_P_y, float* log_P_dur, float* log_prob, void* workspace,
                    size_t workspace_bytes, asr_stream_t stream);

/* Replaces tdt_backward_cuda (tdt.cu:602-704; asr::tdt_backward, tdt_bindings.cpp:32-35).
 * Writes (overwrites) grad_encoder, grad_decoder, grad_joint_W (V,d), grad_joint_W_dur (n_dur,d). */
int asr_tdt_backward(const float* encoder, const float* decoder, const float* joint_W, const float* joint_W_dur,
                     const int32_t* targets, const int32_t* in_lens, const int32_t* tgt_lens,
                     const int32_t* durations, int n_dur, int max_duration, int has_zero, int B, int T, int U,
                     int V, int d, int S, int blank_idx, const double* alpha, const float* log_P_blank,
                     const float* log_P_y, const float* log_P_dur, const float* log_prob, const float* grad_loss,
                     int tf32, float* grad_encoder, float* grad_decoder, float* grad_joint_W,
                     float* grad_joint_W_dur, void* workspace, size_t workspace_bytes, asr_stream_t stream);

/* ------------------------------------------- bf16 activations (*_ex variants)
 *
 * The entry points above with the encoder / decoder activations (and, in the
 * backward, their gradients) of element type act_dtype (asr_dtype_t): bf16 lets a
 * system pass its autocast activations without float32 copies. The tensor-core
 * joint (tf32 != 0) reads bf16 activations directly; the fp32 path reads float32
 * copies that the call makes in its workspace. bf16 gradients are summed in
 * float32 in the workspace and rounded once. Activation rows must be 16-byte
 * aligned for the vector loads (otherwise a scalar path is taken). With act_dtype =
 * ASR_DTYPE_F32 each is identical to its float32 entry point. No counterpart in
 * the reference, whose ops take float32 only (the systems' .float() copies,
 * system/rnnt.py:51, system/tdt.py:59). */
size_t asr_rnnt_workspace_bytes_ex(int B, int T, int U, int V, int d, int tf32, int backward, int act_dtype);
int asr_rnnt_forward_ex(const void* encoder, const void* decoder, int act_dtype, const float* joint_W,
                        const int32_t* targets, const int32_t* in_lens, const int32_t* tgt_lens, int B, int T,
                        int U, int V, int d, int S, int blank_idx, int tf32, float* loss, double* alpha,
                        float* log_P_blank, float* log_P_y, float* log_prob, void* workspace,
                        size_t workspace_bytes, asr_stream_t stream);
int asr_rnnt_backward_ex(const void* encoder, const void* decoder, int act_dtype, const float* joint_W,
                         const int32_t* targets, const int32_t* in_lens, const int32_t* tgt_lens, int B, int T,
                         int U, int V, int d, int S, int blank_idx, const double* alpha, const float* log_P_blank,
                         const float* log_P_y, const float* log_prob, const float* grad_loss, int tf32,
                         void* grad_encoder, void* grad_decoder, float* grad_joint_W, void* workspace,
                         size_t workspace_bytes, asr_stream_t stream);
size_t asr_tdt_workspace_bytes_ex(int B, int T, int U, int V, int n_dur, int d, int tf32, int backward,
                                  int act_dtype);
int asr_tdt_forward_ex(const void* encoder, const void* decoder, int act_dtype, const float* joint_W,
                       const float* joint_W_dur, const int32_t* targets, const int32_t* in_lens,
                       const int32_t* tgt_lens, const int32_t* durations, int n_dur, int max_duration, int has_zero,
                       int B, int T, int U, int V, int d, int S, int blank_idx, float sigma, int tf32, float* loss,
                       double* alpha, float* log_P_blank, float* log_P_y, float* log_P_dur, float* log_prob,
                       void* workspace, size_t workspace_bytes, asr_stream_t stream);
int asr_tdt_backward_ex(const void* encoder, const void* decoder, int act_dtype, const float* joint_W,
                        const float* joint_W_dur, const int32_t* targets, const int32_t* in_lens,
                        const int32_t* tgt_lens, const int32_t* durations, int n_dur, int max_duration, int has_zero,
                        int B, int T, int U, int V, int d, int S, int blank_idx, const double* alpha,
                        const float* log_P_blank, const float* log_P_y, const float* log_P_dur,
                        const float* log_prob, const float* grad_loss, int tf32, void* grad_encoder,
                        void* grad_decoder, float* grad_joint_W, float* grad_joint_W_dur, void* workspace,
                        size_t workspace_bytes, asr_stream_t stream);

/* ---------------------------------------------------- logit stash (*_stash variants)
 *
 * The *_ex entry points with a caller-owned logit stash: the forward keeps the
 * joint's logits of the first lattice nodes that fit in `stash` (compact node
 * order: utterance, frame, label position), and the backward forms d loss /
 * d logits of those nodes in one streaming pass over the stash (about 4 KB of
 * HBM traffic per node at V = 1024) instead of recomputing the logits GEMM
 * (2 * d * (V + n_dur) FLOPs per node). Nodes past the stash are recomputed as
 * in the *_ex backward. A stash row holds each logit minus the row's largest
 * token logit of its vocabulary chunk: fp16 with the bf16 tensor-core joint
 * (tf32 != 0; at most 2^-12 of that difference added to a logit, below the
 * bf16 rounding of the joint's operands for the entries that carry the softmax
 * mass), fp32 in the fp32 mode. The backward must get the same stash (contents
 * untouched), stash_bytes and tf32 as its forward; the backward only reads it,
 * so several backwards over one forward may share it. stash = NULL (or a stash too
 * small for 256 nodes) makes each identical to its *_ex entry point. The stash
 * is used only where both directions run the tensor-core joint. No counterpart
 * in the reference, whose backward always recomputes the logits
 * (src/asr/loss/csrc/rnnt.cu:382-458, tdt.cu:602-704). */

/* Bytes of a stash that holds every node of the capacity B*T*U (n_dur = 0 for
 * RNN-T): ceil256(B*T*U) * (2 or 4 bytes * ceil16(V + n_dur) + 4 bytes per
 * vocabulary chunk) + 512. 0 when the shape does not run the tensor-core joint
 * in both directions (or without a CUDA device). A smaller stash holds the
 * first floor((stash_bytes - 512) / bytes per node) nodes, in whole 256s. */
size_t asr_logit_stash_bytes(int B, int T, int U, int V, int n_dur, int d, int tf32);
int asr_rnnt_forward_stash(const void* encoder, const void* decoder, int act_dtype, const float* joint_W,
                           const int32_t* targets, const int32_t* in_lens, const int32_t* tgt_lens, int B, int T,
                           int U, int V, int d, int S, int blank_idx, int tf32, float* loss, double* alpha,
                           float* log_P_blank, float* log_P_y, float* log_prob, void* stash, size_t stash_bytes,
                           void* workspace, size_t workspace_bytes, asr_stream_t stream);
int asr_rnnt_backward_stash(const void* encoder, const void* decoder, int act_dtype, const float* joint_W,
                            const int32_t* targets, const int32_t* in_lens, const int32_t* tgt_lens, int B, int T,
                            int U, int V, int d, int S, int blank_idx, const double* alpha, const float* log_P_blank,
                            const float* log_P_y, const float* log_prob, const float* grad_loss, int tf32,
                            void* grad_encoder, void* grad_decoder, float* grad_joint_W, const void* stash,
                            size_t stash_bytes, void* workspace, size_t workspace_bytes, asr_stream_t stream);
int asr_tdt_forward_stash(const void* encoder, const void* decoder, int act_dtype, const float* joint_W,
                          const float* joint_W_dur, const int32_t* targets, const int32_t* in_lens,
                          const int32_t* tgt_lens, const int32_t* durations, int n_dur, int max_duration,
                          int has_zero, int B, int T, int U, int V, int d, int S, int blank_idx, float sigma,
                          int tf32, float* loss, double* alpha, float* log_P_blank, float* log_P_y,
                          float* log_P_dur, float* log_prob, void* stash, size_t stash_bytes, void* workspace,
                          size_t workspace_bytes, asr_stream_t stream);
int asr_tdt_backward_stash(const void* encoder, const void* decoder, int act_dtype, const float* joint_W,
                           const float* joint_W_dur, const int32_t* targets, const int32_t* in_lens,
                           const int32_t* tgt_lens, const int32_t* durations, int n_dur, int max_duration,
                           int has_zero, int B, int T, int U, int V, int d, int S, int blank_idx,
                           const double* alpha, const float* log_P_blank, const float* log_P_y,
                           const float* log_P_dur, const float* log_prob, const float* grad_loss, int tf32,
                           void* grad_encoder, void* grad_decoder, float* grad_joint_W, float* grad_joint_W_dur,
                           const void* stash, size_t stash_bytes, void* workspace, size_t workspace_bytes,
                           asr_stream_t stream);

/* Bytes of the scratch array compiled into the library for asr_tdt_forward_noalloc. */
#define ASR_TDT_FORWARD_NOALLOC_SCRATCH_BYTES (4u << 20)

/* asr_tdt_forward without a workspace argument, for callers that cannot allocate
 * device memory (a bare FFI host with no device allocator, a service that reserves
 * all GPU memory at start-up, code where a cudaMalloc would synchronise the device).
 * No counterpart in the reference. Its scratch is a fixed array of
 * ASR_TDT_FORWARD_NOALLOC_SCRATCH_BYTES in device memory, held by every GPU that
 * loads the library; problems whose asr_tdt_workspace_bytes(..., backward = 0)
 * exceed it return ASR_ERR_SCRATCH_LIMIT without launching anything. With
 * tf32 = 0 that workspace is the per-utterance lattice bookkeeping (about 16
 * bytes per utterance); with tf32 = 1 it also holds a bf16 copy of the joint
 * weights (2 * ceil16(V + n_dur) * ceil64(d) bytes) and one bf16 hidden row per
 * lattice node of capacity (2 * ceil64(d) bytes for each of B * T * U nodes), so
 * at V = 1024 + 5 and d = 640 only B * T * U up to about 2,000 nodes fit. The
 * array's device address is looked up on every call in the calling thread's
 * current CUDA context, so any context that has loaded the library works; the
 * first call in a context loads the module there (make it before any stream
 * capture). All calls share the array, so calls that overlap on the GPU race;
 * serialise them. Allocates nothing. */
int asr_tdt_forward_noalloc(const float* encoder, const float* decoder, const float* joint_W,
                            const float* joint_W_dur, const int32_t* targets, const int32_t* in_lens,
                            const int32_t* tgt_lens, const int32_t* durations, int n_dur, int max_duration,
                            int has_zero, int B, int T, int U, int V, int d, int S, int blank_idx, float sigma,
                            int tf32, float* loss, double* alpha, float* log_P_blank, float* log_P_y,
                            float* log_P_dur, float* log_prob, asr_stream_t stream);

/* ------------------------------------------------------- fused CTC head */

/* The CTC system's head and loss in one pass: Linear(RMSNorm(enc)) (reference
 * src/asr/system/ctc.py:21-24: torch.nn.RMSNorm(d) then torch.nn.Linear(d, V),
 * run under bf16 autocast) followed by CTCLoss (src/asr/loss/ctc.py:11-30:
 * log_softmax in fp32, the CTC recursion, blank = 0, zero_infinity), without the
 * (B, T, V) logits, log-probs or their gradient in HBM. No counterpart in the
 * reference, which materialises all three.
 * encoder (B, T, d) float32 or bfloat16 (act_dtype; grad_encoder has the same
 * type); rms_weight (d,); weight (V, d); bias (V,) or NULL; targets (B, S) int32
 * labels in [1, V); in_lens in [1, T]; tgt_lens in [0, S]. The GEMM runs on bf16
 * tcgen05 tensor cores with fp32 accumulation: bf16(RMSNorm(enc)) and bf16(weight,
 * bias), the operands the autocast Linear uses. rms_eps: torch's default is
 * FLT_EPSILON.
 * loss (B,) = -log P(targets | enc), 0 where zero_infinity drops an infeasible
 * utterance (not divided by tgt_lens; CTCLoss divides by tgt_lens.clamp_min(1)).
 * The forward leaves what the backward needs in the workspace: call
 * asr_ctc_head_backward with the same workspace and inputs before reusing it.
 * 2S + 1 <= 1024 and asr_ctc_head_supported(V, d), else ASR_ERR_UNSUPPORTED. */
size_t asr_ctc_head_workspace_bytes(int B, int T, int S, int V, int d, int act_dtype);
int asr_ctc_head_supported(int V, int d);
int asr_ctc_head_forward(const void* encoder, int act_dtype, const float* rms_weight, float rms_eps,
                         const float* weight, const float* bias, const int32_t* targets, const int32_t* in_lens,
                         const int32_t* tgt_lens, int B, int T, int S, int V, int d, int zero_infinity, float* loss,
                         void* workspace, size_t workspace_bytes, asr_stream_t stream);
/* Writes (overwrites) grad_encoder (B, T, d), zero past in_lens; grad_rms_weight
 * (d,); grad_weight (V, d); grad_bias (V,) when bias is given. grad_loss (B,)
 * scales each utterance. */
int asr_ctc_head_backward(const void* encoder, int act_dtype, const float* rms_weight, float rms_eps,
                          const float* weight, const float* bias, const int32_t* targets, const int32_t* in_lens,
                          const int32_t* tgt_lens, int B, int T, int S, int V, int d, int zero_infinity,
                          const float* grad_loss, void* grad_encoder, float* grad_rms_weight, float* grad_weight,
                          float* grad_bias, void* workspace, size_t workspace_bytes, asr_stream_t stream);

/* --------------------------------------------------- CTC prefix beam search */

/* Replaces the reference's CPU op asr::beam_decode (src/asr/decode/csrc/ctc.cpp:46-137;
 * called by src/asr/decode/ctc.py:34-40 beam_decode): prefix beam search over
 * log_probs (B, T, V) float32 on the device, blank = 0, frames t < in_lens[b]
 * (clamped to [0, T]). Writes the best prefix of each utterance to tokens (B, T)
 * int32 (row b holds lengths[b] tokens) and lengths (B,). Same search as the
 * reference: ties between equal scores may resolve differently (the reference's
 * nth_element leaves them unspecified). 1 <= beam_width <= 64 and V <= 8192, else
 * ASR_ERR_UNSUPPORTED. Workspace: asr_ctc_beam_workspace_bytes. */
size_t asr_ctc_beam_workspace_bytes(int B, int T, int beam_width);
int asr_ctc_beam_decode(const float* log_probs, const int32_t* in_lens, int B, int T, int V, int beam_width,
                        int32_t* tokens, int32_t* lengths, void* workspace, size_t workspace_bytes,
                        asr_stream_t stream);

/* ------------------------------------------------ greedy transducer decoding */

/* Batched greedy decoding for RNN-T and TDT. Replaces the per-utterance,
 * per-symbol joint calls of the reference decoders (src/asr/decode/rnnt.py:12-37
 * greedy_decode; src/asr/decode/tdt.py:14-62 greedy_decode), whose joint is
 * Linear(tanh(enc_t + pred_u)) without bias (src/asr/system/rnnt.py:29-34,
 * src/asr/system/tdt.py:31-43). The reference has no C interface for decoding;
 * these entry points are driven by a host loop (asr_b200/decode/_greedy.py):
 *
 *   asr_greedy_pack_weights(W -> Wt); asr_greedy_init(state, prefix);
 *   pred[b] = predictor output for the prefix [<sos>], every b;
 *   active = all b;
 *   loop: asr_greedy_scan(active, ...); read report (B,);
 *         active = the b of the list with report[b] > 0 or == -2; stop when
 *         empty; for every b with report[b] = L > 0, pred[b] = predictor
 *         output at position L-1 of prefix[b, :L].
 *
 * Buffers, all device memory, row-major:
 *   state  (B, 4) int32   per utterance: frame t, symbols emitted at t, hypothesis
 *                         length, number of recorded durations;
 *   prefix (B, hyp_cap+1) int64  <sos> followed by the emitted tokens;
 *   durs   (B, dur_cap) int32   TDT only: the argmax duration of every step,
 *                         blanks included (the reference's second return value);
 *   report (B,) int32     after a scan: L = prefix length when utterance b emitted a
 *                         token and needs a new predictor output, 0 when it has
 *                         finished, -2 when it stopped at max_windows (scan it
 *                         again, pred unchanged), -1 when hyp_cap or dur_cap was
 *                         too small.
 * hyp_cap = dur_cap = T * max_symbols_per_frame can never overflow. */

/* joint_Wt (d, ldw) = transpose of joint_W (V, d), columns V..ldw-1 zeroed.
 * ldw >= V, a multiple of 4; joint_Wt 16-byte aligned. */
int asr_greedy_pack_weights(const float* joint_W, int V, int d, float* joint_Wt, int ldw, asr_stream_t stream);

/* Zeroes state and fills prefix with <sos> = sos_id: prefix[b, 0] is the start
 * token, and positions past a hypothesis hold sos_id (a valid token id when a
 * predictor is run on right-padded prefixes). */
int asr_greedy_init(int32_t* state, int64_t* prefix, int B, int hyp_cap, int sos_id, asr_stream_t stream);

/* Advances each utterance of the active list (n_active indices into the batch;
 * active = NULL: all B) from its state to its next emitted token or to its end
 * (frame t >= in_lens[b]) with the predictor output pred (B, d); report[b] is
 * written for those utterances only. Utterances that reported 0 are finished and
 * may be left out of later lists; a finished utterance in the list reports 0
 * again.
 * encoder (B, T, d) float32; joint_Wt from asr_greedy_pack_weights;
 * joint_W_dur (n_dur, d) float32 selects TDT when n_dur > 0 (duration value =
 * argmax index, the reference's durations = range(max_duration + 1)); n_dur = 0
 * and joint_W_dur = NULL select RNN-T. Ties take the lowest index and NaN counts
 * as the maximum (torch.argmax). max_symbols_per_frame <= 0 finishes every
 * utterance without emitting, as the reference's empty per-frame loop does.
 * in_lens outside [0, T] are clamped. d <= 2048 and n_dur <= 64, else
 * ASR_ERR_UNSUPPORTED. max_windows > 0 bounds the frames one utterance scans in
 * this call to max_windows windows of 8 frames: an utterance that reaches it
 * without emitting or finishing reports -2 and continues, from its saved state
 * and with the same pred row, when it is next in the active list (0: no bound). */
int asr_greedy_scan(const float* encoder, const float* pred, const float* joint_Wt, int ldw,
                    const float* joint_W_dur, const int32_t* in_lens, const int32_t* active, int n_active,
                    int32_t* state, int64_t* prefix, int32_t* durs, int32_t* report, int B, int T, int d, int V,
                    int n_dur, int blank_idx, int max_symbols_per_frame, int hyp_cap, int dur_cap,
                    int max_windows, asr_stream_t stream);

/* ----------------------------------------------------------- diagnostics */

/* Copies the device status word of a workspace used by the last call on it
 * into *clamped (1 = some length was out of range and was clamped). Synchronises
 * `stream`. Intended for debugging; the hot path never calls it. */
int asr_workspace_status(const void* workspace, int B, int* clamped, asr_stream_t stream);

/* Joint-network path a call takes: 1 = tcgen05 tensor cores, 0 = fp32 SIMT.
 * With tf32 = 1 the tensor-core path uses bf16 operands; with tf32 = 0 it keeps
 * fp32 accuracy by splitting every operand into two bf16 parts and summing three
 * products (hi*hi + lo*hi + hi*lo) in fp32. ASR_B200_FP32_SIMT=1 in the
 * environment sends tf32 = 0 calls to the SIMT path instead. */
int asr_joint_path(int tf32, int V, int n_dur, int d);

/* Per-kernel device timing of this library's own launches: while enabled, every
 * kernel launch is bracketed by CUDA events on its stream. Off by default; the
 * overhead when off is one flag test per launch. No counterpart in the reference. */
int asr_profiler_enable(int on);

/* Waits for the recorded events and writes "<kernel> <launches> <total_ms>" lines
 * into buf (NUL-terminated, truncated to len). Returns the full report length, or a
 * negative asr_status_t. clear != 0 drops the records afterwards. */
int asr_profiler_report(char* buf, size_t len, int clear);

#ifdef __cplusplus
}
#endif

#endif /* ASR_B200_H_ */
