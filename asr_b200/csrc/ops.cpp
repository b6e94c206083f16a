// PyTorch stable-ABI operator shim: registers the six `asr::*` ops with the
// exact schemas of the reference (src/asr/loss/csrc/ctc_bindings.cpp:16-22,
// rnnt_bindings.cpp:22-30, tdt_bindings.cpp:26-36), so the reference's Python
// loss modules run on this library unchanged. Each op validates its tensors
// like the reference (CUDA, contiguous, float32 / int32; the transducer ops also
// take bf16 encoder / decoder activations and return bf16 gradients for them),
// allocates outputs and
// workspace through the torch caching allocator, and calls the C ABI of
// include/asr_b200.h on the current stream of the input's device.
#include <torch/csrc/inductor/aoti_torch/c/shim.h>
#include <torch/csrc/stable/accelerator.h>
#include <torch/csrc/stable/library.h>
#include <torch/csrc/stable/ops.h>
#include <torch/csrc/stable/tensor.h>

#include <algorithm>
#include <tuple>

#include "asr_b200.h"

using torch::stable::Tensor;
using torch::headeronly::ScalarType;

namespace {

#define ASR_CHECK_F32(x)                                                                                   \
    STD_TORCH_CHECK(x.is_cuda(), #x " must be a CUDA tensor");                                             \
    STD_TORCH_CHECK(x.is_contiguous(), #x " must be contiguous");                                          \
    STD_TORCH_CHECK(x.scalar_type() == ScalarType::Float, #x " must be float32")

#define ASR_CHECK_F64(x)                                                                                   \
    STD_TORCH_CHECK(x.is_cuda(), #x " must be a CUDA tensor");                                             \
    STD_TORCH_CHECK(x.is_contiguous(), #x " must be contiguous");                                          \
    STD_TORCH_CHECK(x.scalar_type() == ScalarType::Double, #x " must be the float64 forward variable of the forward op")

#define ASR_CHECK_I32(x)                                                                                   \
    STD_TORCH_CHECK(x.is_cuda(), #x " must be a CUDA tensor");                                             \
    STD_TORCH_CHECK(x.is_contiguous(), #x " must be contiguous");                                          \
    STD_TORCH_CHECK(x.scalar_type() == ScalarType::Int, #x " must be int")

// Encoder / decoder activations: float32 (the reference's contract) or bf16 (a
// system's autocast activations, no float32 copies); both the same type.
int act_dtype(const Tensor& encoder, const Tensor& decoder) {
    STD_TORCH_CHECK(encoder.is_cuda() && decoder.is_cuda(), "encoder and decoder must be CUDA tensors");
    STD_TORCH_CHECK(encoder.is_contiguous() && decoder.is_contiguous(), "encoder and decoder must be contiguous");
    const ScalarType t = encoder.scalar_type();
    STD_TORCH_CHECK(t == ScalarType::Float || t == ScalarType::BFloat16, "encoder must be float32 or bfloat16");
    STD_TORCH_CHECK(decoder.scalar_type() == t, "decoder must have the encoder's dtype");
    return t == ScalarType::BFloat16 ? ASR_DTYPE_BF16 : ASR_DTYPE_F32;
}

asr_stream_t current_stream(const Tensor& t) {
    void* s = nullptr;
    TORCH_ERROR_CODE_CHECK(aoti_torch_get_current_cuda_stream(t.get_device_index(), &s));
    return reinterpret_cast<asr_stream_t>(s);
}

void check_rc(int rc, const char* op) { STD_TORCH_CHECK(rc == ASR_OK, op, ": ", asr_status_string(rc)); }

Tensor workspace(const Tensor& like, size_t bytes) {
    return torch::stable::new_empty(like, {(int64_t)(bytes > 0 ? bytes : 1)}, ScalarType::Byte);
}

int dim(const Tensor& t, int i) { return (int)t.sizes()[i]; }

// Logit stash of the *_stash ops: the bytes that hold every node of the
// capacity, at most `budget`; a 1-byte placeholder (no stash) when the budget is
// 0 or the shape does not run the tensor-core joint.
Tensor stash_tensor(const Tensor& like, size_t full_bytes, int64_t budget) {
    const size_t bytes = budget > 0 ? std::min(full_bytes, (size_t)budget) : 0;
    return workspace(like, bytes > 512 ? bytes : 0);
}

int target_cols(const Tensor& targets) { return targets.dim() >= 2 ? dim(targets, 1) : 0; }

// --------------------------------------------------------------------- CTC

std::tuple<Tensor, Tensor> ctc_alpha(const Tensor& log_probs, const Tensor& targets, const Tensor& in_lens,
                                     const Tensor& tgt_lens) {
    ASR_CHECK_F32(log_probs);
    ASR_CHECK_I32(targets);
    ASR_CHECK_I32(in_lens);
    ASR_CHECK_I32(tgt_lens);
    torch::stable::accelerator::DeviceGuard guard(log_probs.get_device_index());
    const int B = dim(log_probs, 0), T = dim(log_probs, 1), V = dim(log_probs, 2), S = target_cols(targets);
    Tensor alpha = torch::stable::new_empty(log_probs, {B, T, 2 * S + 1}, ScalarType::Double);
    Tensor log_Z = torch::stable::new_empty(log_probs, {B});
    check_rc(asr_ctc_alpha(log_probs.const_data_ptr<float>(), targets.const_data_ptr<int32_t>(),
                           in_lens.const_data_ptr<int32_t>(), tgt_lens.const_data_ptr<int32_t>(), B, T, V, S,
                           alpha.mutable_data_ptr<double>(), log_Z.mutable_data_ptr<float>(),
                           current_stream(log_probs)),
             "asr::ctc_alpha");
    return {alpha, log_Z};
}

Tensor ctc_grad(const Tensor& alpha, const Tensor& log_Z, const Tensor& log_probs, const Tensor& targets,
                const Tensor& in_lens, const Tensor& tgt_lens, const Tensor& grad_loss, bool zero_infinity) {
    ASR_CHECK_F64(alpha);
    ASR_CHECK_F32(log_Z);
    ASR_CHECK_F32(log_probs);
    ASR_CHECK_I32(targets);
    ASR_CHECK_I32(in_lens);
    ASR_CHECK_I32(tgt_lens);
    ASR_CHECK_F32(grad_loss);
    torch::stable::accelerator::DeviceGuard guard(log_probs.get_device_index());
    const int B = dim(log_probs, 0), T = dim(log_probs, 1), V = dim(log_probs, 2), S = target_cols(targets);
    Tensor grad = torch::stable::new_empty(log_probs, {B, T, V});
    check_rc(asr_ctc_grad(alpha.const_data_ptr<double>(), log_Z.const_data_ptr<float>(),
                          log_probs.const_data_ptr<float>(), targets.const_data_ptr<int32_t>(),
                          in_lens.const_data_ptr<int32_t>(), tgt_lens.const_data_ptr<int32_t>(),
                          grad_loss.const_data_ptr<float>(), zero_infinity ? 1 : 0, B, T, V, S,
                          grad.mutable_data_ptr<float>(), current_stream(log_probs)),
             "asr::ctc_grad");
    return grad;
}

// -------------------------------------------------------------------- RNN-T

std::tuple<Tensor, Tensor, Tensor, Tensor, Tensor, Tensor> rnnt_forward_impl(
    const Tensor& encoder, const Tensor& decoder, const Tensor& joint_W, const Tensor& targets, const Tensor& in_lens,
    const Tensor& tgt_lens, int64_t blank_idx, int64_t tf32, int64_t stash_budget) {
    const int act = act_dtype(encoder, decoder);
    ASR_CHECK_F32(joint_W);
    ASR_CHECK_I32(targets);
    ASR_CHECK_I32(in_lens);
    ASR_CHECK_I32(tgt_lens);
    torch::stable::accelerator::DeviceGuard guard(encoder.get_device_index());
    const int B = dim(encoder, 0), T = dim(encoder, 1), d = dim(encoder, 2), U = dim(decoder, 1);
    const int V = dim(joint_W, 0), S = target_cols(targets);
    STD_TORCH_CHECK(dim(decoder, 0) == B && dim(decoder, 2) == d && dim(joint_W, 1) == d, "rnnt_forward: shape mismatch");
    Tensor loss = torch::stable::new_empty(encoder, {B}, ScalarType::Float);
    Tensor log_prob = torch::stable::new_empty(encoder, {B}, ScalarType::Float);
    Tensor alpha = torch::stable::new_empty(encoder, {B, T, U}, ScalarType::Double);
    Tensor log_P_blank = torch::stable::new_empty(encoder, {2, B, T, U}, ScalarType::Float);
    Tensor log_P_y = torch::stable::new_empty(encoder, {B, T, U}, ScalarType::Float);
    Tensor stash = stash_tensor(encoder, asr_logit_stash_bytes(B, T, U, V, 0, d, (int)tf32), stash_budget);
    const size_t wsb = asr_rnnt_workspace_bytes_ex(B, T, U, V, d, (int)tf32, 0, act);
    Tensor ws = workspace(encoder, wsb);
    check_rc(asr_rnnt_forward_stash(encoder.const_data_ptr(), decoder.const_data_ptr(), act,
                                    joint_W.const_data_ptr<float>(), targets.const_data_ptr<int32_t>(),
                                    in_lens.const_data_ptr<int32_t>(), tgt_lens.const_data_ptr<int32_t>(), B, T, U, V,
                                    d, S, (int)blank_idx, (int)tf32, loss.mutable_data_ptr<float>(),
                                    alpha.mutable_data_ptr<double>(), log_P_blank.mutable_data_ptr<float>(),
                                    log_P_y.mutable_data_ptr<float>(), log_prob.mutable_data_ptr<float>(),
                                    stash.mutable_data_ptr(), (size_t)stash.numel(), ws.mutable_data_ptr(), wsb,
                                    current_stream(encoder)),
             "asr::rnnt_forward");
    return {loss, alpha, log_P_blank, log_P_y, log_prob, stash};
}

std::tuple<Tensor, Tensor, Tensor, Tensor, Tensor> rnnt_forward(const Tensor& encoder, const Tensor& decoder,
                                                                const Tensor& joint_W, const Tensor& targets,
                                                                const Tensor& in_lens, const Tensor& tgt_lens,
                                                                int64_t blank_idx, int64_t tf32) {
    auto [loss, alpha, log_P_blank, log_P_y, log_prob, stash] =
        rnnt_forward_impl(encoder, decoder, joint_W, targets, in_lens, tgt_lens, blank_idx, tf32, 0);
    return {loss, alpha, log_P_blank, log_P_y, log_prob};
}

// rnnt_forward that also returns the logit stash (at most stash_budget bytes)
// for rnnt_backward_stash.
std::tuple<Tensor, Tensor, Tensor, Tensor, Tensor, Tensor> rnnt_forward_stash(
    const Tensor& encoder, const Tensor& decoder, const Tensor& joint_W, const Tensor& targets, const Tensor& in_lens,
    const Tensor& tgt_lens, int64_t blank_idx, int64_t tf32, int64_t stash_budget) {
    return rnnt_forward_impl(encoder, decoder, joint_W, targets, in_lens, tgt_lens, blank_idx, tf32, stash_budget);
}

std::tuple<Tensor, Tensor, Tensor> rnnt_backward_impl(const Tensor& encoder, const Tensor& decoder,
                                                      const Tensor& joint_W, const Tensor& targets,
                                                      const Tensor& in_lens, const Tensor& tgt_lens, int64_t blank_idx,
                                                      const Tensor& alpha, const Tensor& log_P_blank,
                                                      const Tensor& log_P_y, const Tensor& log_prob,
                                                      const Tensor& grad_loss, int64_t tf32, const Tensor* stash) {
    const int act = act_dtype(encoder, decoder);
    ASR_CHECK_F32(joint_W);
    ASR_CHECK_I32(targets);
    ASR_CHECK_I32(in_lens);
    ASR_CHECK_I32(tgt_lens);
    ASR_CHECK_F64(alpha);
    ASR_CHECK_F32(log_P_blank);
    ASR_CHECK_F32(log_P_y);
    ASR_CHECK_F32(log_prob);
    ASR_CHECK_F32(grad_loss);
    torch::stable::accelerator::DeviceGuard guard(encoder.get_device_index());
    const int B = dim(encoder, 0), T = dim(encoder, 1), d = dim(encoder, 2), U = dim(decoder, 1);
    const int V = dim(joint_W, 0), S = target_cols(targets);
    STD_TORCH_CHECK(log_P_blank.numel() == 2LL * B * T * U, "rnnt_backward: log_P_blank is not a forward output");
    Tensor g_enc = torch::stable::new_empty(encoder, {B, T, d});
    Tensor g_dec = torch::stable::new_empty(encoder, {B, U, d});
    Tensor g_W = torch::stable::new_empty(joint_W, {V, d});
    const size_t wsb = asr_rnnt_workspace_bytes_ex(B, T, U, V, d, (int)tf32, 1, act);
    Tensor ws = workspace(encoder, wsb);
    check_rc(asr_rnnt_backward_stash(encoder.const_data_ptr(), decoder.const_data_ptr(), act,
                                     joint_W.const_data_ptr<float>(), targets.const_data_ptr<int32_t>(),
                                     in_lens.const_data_ptr<int32_t>(), tgt_lens.const_data_ptr<int32_t>(), B, T, U, V,
                                     d, S, (int)blank_idx, alpha.const_data_ptr<double>(),
                                     log_P_blank.const_data_ptr<float>(), log_P_y.const_data_ptr<float>(),
                                     log_prob.const_data_ptr<float>(), grad_loss.const_data_ptr<float>(), (int)tf32,
                                     g_enc.mutable_data_ptr(), g_dec.mutable_data_ptr(), g_W.mutable_data_ptr<float>(),
                                     stash ? stash->const_data_ptr() : nullptr, stash ? (size_t)stash->numel() : 0,
                                     ws.mutable_data_ptr(), wsb, current_stream(encoder)),
             "asr::rnnt_backward");
    return {g_enc, g_dec, g_W};
}

std::tuple<Tensor, Tensor, Tensor> rnnt_backward(const Tensor& encoder, const Tensor& decoder, const Tensor& joint_W,
                                                 const Tensor& targets, const Tensor& in_lens,
                                                 const Tensor& tgt_lens, int64_t blank_idx, const Tensor& alpha,
                                                 const Tensor& log_P_blank, const Tensor& log_P_y,
                                                 const Tensor& log_prob, const Tensor& grad_loss, int64_t tf32) {
    return rnnt_backward_impl(encoder, decoder, joint_W, targets, in_lens, tgt_lens, blank_idx, alpha, log_P_blank,
                              log_P_y, log_prob, grad_loss, tf32, nullptr);
}

// rnnt_backward over the logit stash of rnnt_forward_stash (same tf32).
std::tuple<Tensor, Tensor, Tensor> rnnt_backward_stash(const Tensor& encoder, const Tensor& decoder,
                                                       const Tensor& joint_W, const Tensor& targets,
                                                       const Tensor& in_lens, const Tensor& tgt_lens,
                                                       int64_t blank_idx, const Tensor& alpha,
                                                       const Tensor& log_P_blank, const Tensor& log_P_y,
                                                       const Tensor& log_prob, const Tensor& grad_loss, int64_t tf32,
                                                       const Tensor& stash) {
    STD_TORCH_CHECK(stash.is_cuda() && stash.is_contiguous() && stash.scalar_type() == ScalarType::Byte,
                    "rnnt_backward_stash: stash is not a stash of rnnt_forward_stash");
    return rnnt_backward_impl(encoder, decoder, joint_W, targets, in_lens, tgt_lens, blank_idx, alpha, log_P_blank,
                              log_P_y, log_prob, grad_loss, tf32, &stash);
}

// ---------------------------------------------------------------------- TDT

std::tuple<Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor> tdt_forward_impl(
    const Tensor& encoder, const Tensor& decoder, const Tensor& joint_W, const Tensor& joint_W_dur,
    const Tensor& targets, const Tensor& in_lens, const Tensor& tgt_lens, const Tensor& durations,
    int64_t max_duration, int64_t has_zero, int64_t blank_idx, double sigma, int64_t tf32, int64_t stash_budget) {
    const int act = act_dtype(encoder, decoder);
    ASR_CHECK_F32(joint_W);
    ASR_CHECK_F32(joint_W_dur);
    ASR_CHECK_I32(targets);
    ASR_CHECK_I32(in_lens);
    ASR_CHECK_I32(tgt_lens);
    ASR_CHECK_I32(durations);
    torch::stable::accelerator::DeviceGuard guard(encoder.get_device_index());
    const int B = dim(encoder, 0), T = dim(encoder, 1), d = dim(encoder, 2), U = dim(decoder, 1);
    const int V = dim(joint_W, 0), Dn = dim(joint_W_dur, 0), S = target_cols(targets);
    STD_TORCH_CHECK(durations.numel() == Dn, "tdt_forward: durations must have one entry per joint_W_dur row");
    Tensor loss = torch::stable::new_empty(encoder, {B}, ScalarType::Float);
    Tensor log_prob = torch::stable::new_empty(encoder, {B}, ScalarType::Float);
    Tensor alpha = torch::stable::new_empty(encoder, {B, T + 1, U}, ScalarType::Double);
    Tensor log_P_blank = torch::stable::new_empty(encoder, {2, B, T, U}, ScalarType::Float);
    Tensor log_P_y = torch::stable::new_empty(encoder, {B, T, U}, ScalarType::Float);
    Tensor log_P_dur = torch::stable::new_empty(encoder, {B, T, U, Dn}, ScalarType::Float);
    Tensor stash = stash_tensor(encoder, asr_logit_stash_bytes(B, T, U, V, Dn, d, (int)tf32), stash_budget);
    const size_t wsb = asr_tdt_workspace_bytes_ex(B, T, U, V, Dn, d, (int)tf32, 0, act);
    Tensor ws = workspace(encoder, wsb);
    check_rc(asr_tdt_forward_stash(encoder.const_data_ptr(), decoder.const_data_ptr(), act,
                                   joint_W.const_data_ptr<float>(), joint_W_dur.const_data_ptr<float>(),
                                   targets.const_data_ptr<int32_t>(), in_lens.const_data_ptr<int32_t>(),
                                   tgt_lens.const_data_ptr<int32_t>(), durations.const_data_ptr<int32_t>(), Dn,
                                   (int)max_duration, (int)has_zero, B, T, U, V, d, S, (int)blank_idx, (float)sigma,
                                   (int)tf32, loss.mutable_data_ptr<float>(), alpha.mutable_data_ptr<double>(),
                                   log_P_blank.mutable_data_ptr<float>(), log_P_y.mutable_data_ptr<float>(),
                                   log_P_dur.mutable_data_ptr<float>(), log_prob.mutable_data_ptr<float>(),
                                   stash.mutable_data_ptr(), (size_t)stash.numel(), ws.mutable_data_ptr(), wsb,
                                   current_stream(encoder)),
             "asr::tdt_forward");
    return {loss, alpha, log_P_blank, log_P_y, log_P_dur, log_prob, stash};
}

std::tuple<Tensor, Tensor, Tensor, Tensor, Tensor, Tensor> tdt_forward(
    const Tensor& encoder, const Tensor& decoder, const Tensor& joint_W, const Tensor& joint_W_dur,
    const Tensor& targets, const Tensor& in_lens, const Tensor& tgt_lens, const Tensor& durations,
    int64_t max_duration, int64_t has_zero, int64_t blank_idx, double sigma, int64_t tf32) {
    auto [loss, alpha, log_P_blank, log_P_y, log_P_dur, log_prob, stash] =
        tdt_forward_impl(encoder, decoder, joint_W, joint_W_dur, targets, in_lens, tgt_lens, durations, max_duration,
                         has_zero, blank_idx, sigma, tf32, 0);
    return {loss, alpha, log_P_blank, log_P_y, log_P_dur, log_prob};
}

// tdt_forward that also returns the logit stash (at most stash_budget bytes)
// for tdt_backward_stash.
std::tuple<Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor> tdt_forward_stash(
    const Tensor& encoder, const Tensor& decoder, const Tensor& joint_W, const Tensor& joint_W_dur,
    const Tensor& targets, const Tensor& in_lens, const Tensor& tgt_lens, const Tensor& durations,
    int64_t max_duration, int64_t has_zero, int64_t blank_idx, double sigma, int64_t tf32, int64_t stash_budget) {
    return tdt_forward_impl(encoder, decoder, joint_W, joint_W_dur, targets, in_lens, tgt_lens, durations,
                            max_duration, has_zero, blank_idx, sigma, tf32, stash_budget);
}

std::tuple<Tensor, Tensor, Tensor, Tensor> tdt_backward_impl(
    const Tensor& encoder, const Tensor& decoder, const Tensor& joint_W, const Tensor& joint_W_dur,
    const Tensor& targets, const Tensor& in_lens, const Tensor& tgt_lens, const Tensor& durations,
    int64_t max_duration, int64_t has_zero, int64_t blank_idx, const Tensor& alpha, const Tensor& log_P_blank,
    const Tensor& log_P_y, const Tensor& log_P_dur, const Tensor& log_prob, const Tensor& grad_loss, int64_t tf32,
    const Tensor* stash) {
    const int act = act_dtype(encoder, decoder);
    ASR_CHECK_F32(joint_W);
    ASR_CHECK_F32(joint_W_dur);
    ASR_CHECK_I32(targets);
    ASR_CHECK_I32(in_lens);
    ASR_CHECK_I32(tgt_lens);
    ASR_CHECK_I32(durations);
    ASR_CHECK_F64(alpha);
    ASR_CHECK_F32(log_P_blank);
    ASR_CHECK_F32(log_P_y);
    ASR_CHECK_F32(log_P_dur);
    ASR_CHECK_F32(log_prob);
    ASR_CHECK_F32(grad_loss);
    torch::stable::accelerator::DeviceGuard guard(encoder.get_device_index());
    const int B = dim(encoder, 0), T = dim(encoder, 1), d = dim(encoder, 2), U = dim(decoder, 1);
    const int V = dim(joint_W, 0), Dn = dim(joint_W_dur, 0), S = target_cols(targets);
    STD_TORCH_CHECK(log_P_blank.numel() == 2LL * B * T * U, "tdt_backward: log_P_blank is not a forward output");
    Tensor g_enc = torch::stable::new_empty(encoder, {B, T, d});
    Tensor g_dec = torch::stable::new_empty(encoder, {B, U, d});
    Tensor g_W = torch::stable::new_empty(joint_W, {V, d});
    Tensor g_Wd = torch::stable::new_empty(joint_W_dur, {Dn, d});
    const size_t wsb = asr_tdt_workspace_bytes_ex(B, T, U, V, Dn, d, (int)tf32, 1, act);
    Tensor ws = workspace(encoder, wsb);
    check_rc(asr_tdt_backward_stash(encoder.const_data_ptr(), decoder.const_data_ptr(), act,
                                    joint_W.const_data_ptr<float>(), joint_W_dur.const_data_ptr<float>(),
                                    targets.const_data_ptr<int32_t>(), in_lens.const_data_ptr<int32_t>(),
                                    tgt_lens.const_data_ptr<int32_t>(), durations.const_data_ptr<int32_t>(), Dn,
                                    (int)max_duration, (int)has_zero, B, T, U, V, d, S, (int)blank_idx,
                                    alpha.const_data_ptr<double>(), log_P_blank.const_data_ptr<float>(),
                                    log_P_y.const_data_ptr<float>(), log_P_dur.const_data_ptr<float>(),
                                    log_prob.const_data_ptr<float>(), grad_loss.const_data_ptr<float>(), (int)tf32,
                                    g_enc.mutable_data_ptr(), g_dec.mutable_data_ptr(), g_W.mutable_data_ptr<float>(),
                                    g_Wd.mutable_data_ptr<float>(), stash ? stash->const_data_ptr() : nullptr,
                                    stash ? (size_t)stash->numel() : 0, ws.mutable_data_ptr(), wsb,
                                    current_stream(encoder)),
             "asr::tdt_backward");
    return {g_enc, g_dec, g_W, g_Wd};
}

std::tuple<Tensor, Tensor, Tensor, Tensor> tdt_backward(
    const Tensor& encoder, const Tensor& decoder, const Tensor& joint_W, const Tensor& joint_W_dur,
    const Tensor& targets, const Tensor& in_lens, const Tensor& tgt_lens, const Tensor& durations,
    int64_t max_duration, int64_t has_zero, int64_t blank_idx, const Tensor& alpha, const Tensor& log_P_blank,
    const Tensor& log_P_y, const Tensor& log_P_dur, const Tensor& log_prob, const Tensor& grad_loss, int64_t tf32) {
    return tdt_backward_impl(encoder, decoder, joint_W, joint_W_dur, targets, in_lens, tgt_lens, durations,
                             max_duration, has_zero, blank_idx, alpha, log_P_blank, log_P_y, log_P_dur, log_prob,
                             grad_loss, tf32, nullptr);
}

// tdt_backward over the logit stash of tdt_forward_stash (same tf32).
std::tuple<Tensor, Tensor, Tensor, Tensor> tdt_backward_stash(
    const Tensor& encoder, const Tensor& decoder, const Tensor& joint_W, const Tensor& joint_W_dur,
    const Tensor& targets, const Tensor& in_lens, const Tensor& tgt_lens, const Tensor& durations,
    int64_t max_duration, int64_t has_zero, int64_t blank_idx, const Tensor& alpha, const Tensor& log_P_blank,
    const Tensor& log_P_y, const Tensor& log_P_dur, const Tensor& log_prob, const Tensor& grad_loss, int64_t tf32,
    const Tensor& stash) {
    STD_TORCH_CHECK(stash.is_cuda() && stash.is_contiguous() && stash.scalar_type() == ScalarType::Byte,
                    "tdt_backward_stash: stash is not a stash of tdt_forward_stash");
    return tdt_backward_impl(encoder, decoder, joint_W, joint_W_dur, targets, in_lens, tgt_lens, durations,
                             max_duration, has_zero, blank_idx, alpha, log_P_blank, log_P_y, log_P_dur, log_prob,
                             grad_loss, tf32, &stash);
}

}  // namespace

STABLE_TORCH_LIBRARY(asr, m) {
    m.def("ctc_alpha(Tensor log_probs, Tensor targets, Tensor in_lens, Tensor tgt_lens) -> (Tensor, Tensor)");
    m.def(
        "ctc_grad(Tensor alpha, Tensor log_Z, Tensor log_probs, Tensor targets, Tensor in_lens, Tensor tgt_lens, "
        "Tensor grad_loss, bool zero_infinity) -> Tensor");
    m.def(
        "rnnt_forward(Tensor encoder, Tensor decoder, Tensor joint_W, Tensor targets, Tensor in_lens, "
        "Tensor tgt_lens, int blank_idx, int tf32) -> (Tensor, Tensor, Tensor, Tensor, Tensor)");
    m.def(
        "rnnt_backward(Tensor encoder, Tensor decoder, Tensor joint_W, Tensor targets, Tensor in_lens, "
        "Tensor tgt_lens, int blank_idx, Tensor alpha, Tensor log_P_blank, Tensor log_P_y, Tensor log_prob, "
        "Tensor grad_loss, int tf32) -> (Tensor, Tensor, Tensor)");
    m.def(
        "tdt_forward(Tensor encoder, Tensor decoder, Tensor joint_W, Tensor joint_W_dur, Tensor targets, "
        "Tensor in_lens, Tensor tgt_lens, Tensor durations, int max_duration, int has_zero, int blank_idx, "
        "float sigma, int tf32) -> (Tensor, Tensor, Tensor, Tensor, Tensor, Tensor)");
    m.def(
        "tdt_backward(Tensor encoder, Tensor decoder, Tensor joint_W, Tensor joint_W_dur, Tensor targets, "
        "Tensor in_lens, Tensor tgt_lens, Tensor durations, int max_duration, int has_zero, int blank_idx, "
        "Tensor alpha, Tensor log_P_blank, Tensor log_P_y, Tensor log_P_dur, Tensor log_prob, Tensor grad_loss, "
        "int tf32) -> (Tensor, Tensor, Tensor, Tensor)");
}

// Ops of this library beside the reference's: the transducer ops with a logit
// stash (asr_b200.loss uses them; the reference-schema ops above recompute).
STABLE_TORCH_LIBRARY_FRAGMENT(asr, m) {
    m.def(
        "rnnt_forward_stash(Tensor encoder, Tensor decoder, Tensor joint_W, Tensor targets, Tensor in_lens, "
        "Tensor tgt_lens, int blank_idx, int tf32, int stash_budget) -> (Tensor, Tensor, Tensor, Tensor, Tensor, "
        "Tensor)");
    m.def(
        "rnnt_backward_stash(Tensor encoder, Tensor decoder, Tensor joint_W, Tensor targets, Tensor in_lens, "
        "Tensor tgt_lens, int blank_idx, Tensor alpha, Tensor log_P_blank, Tensor log_P_y, Tensor log_prob, "
        "Tensor grad_loss, int tf32, Tensor stash) -> (Tensor, Tensor, Tensor)");
    m.def(
        "tdt_forward_stash(Tensor encoder, Tensor decoder, Tensor joint_W, Tensor joint_W_dur, Tensor targets, "
        "Tensor in_lens, Tensor tgt_lens, Tensor durations, int max_duration, int has_zero, int blank_idx, "
        "float sigma, int tf32, int stash_budget) -> (Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor)");
    m.def(
        "tdt_backward_stash(Tensor encoder, Tensor decoder, Tensor joint_W, Tensor joint_W_dur, Tensor targets, "
        "Tensor in_lens, Tensor tgt_lens, Tensor durations, int max_duration, int has_zero, int blank_idx, "
        "Tensor alpha, Tensor log_P_blank, Tensor log_P_y, Tensor log_P_dur, Tensor log_prob, Tensor grad_loss, "
        "int tf32, Tensor stash) -> (Tensor, Tensor, Tensor, Tensor)");
}

STABLE_TORCH_LIBRARY_IMPL(asr, CUDA, m) {
    m.impl("rnnt_forward_stash", TORCH_BOX(&rnnt_forward_stash));
    m.impl("rnnt_backward_stash", TORCH_BOX(&rnnt_backward_stash));
    m.impl("tdt_forward_stash", TORCH_BOX(&tdt_forward_stash));
    m.impl("tdt_backward_stash", TORCH_BOX(&tdt_backward_stash));
    m.impl("ctc_alpha", TORCH_BOX(&ctc_alpha));
    m.impl("ctc_grad", TORCH_BOX(&ctc_grad));
    m.impl("rnnt_forward", TORCH_BOX(&rnnt_forward));
    m.impl("rnnt_backward", TORCH_BOX(&rnnt_backward));
    m.impl("tdt_forward", TORCH_BOX(&tdt_forward));
    m.impl("tdt_backward", TORCH_BOX(&tdt_backward));
}
