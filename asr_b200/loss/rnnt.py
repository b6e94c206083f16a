"""RNN-T loss on the B200 kernels (interface of reference src/asr/loss/rnnt.py:11-128)."""

from dataclasses import dataclass

import torch

from asr_b200 import _lib

_lib.load_ops()


class RNNTLossFn(torch.autograd.Function):
    """Fused joint network + RNN-T loss with an exact analytic backward.

    The joint ``tanh(enc + dec) @ joint_W.T`` and its log-softmax run inside the
    kernels, so the (B, T, U, V) logits are never materialised in fp32; the
    forward keeps them (fp16, or fp32 in the fp32 mode) in a stash of at most
    ``asr_b200._lib.logit_stash_budget()`` bytes for the backward, which
    recomputes the logits of nodes past it. ``tf32`` selects the bf16
    tensor-core joint (fp32 accumulation); the default is fp32-exact.
    """

    @staticmethod
    def forward(ctx, encoder, decoder, joint_W, in_lens, tgt_lens, targets, blank_idx, tf32):
        targets = targets.int()
        in_lens = in_lens.int()
        tgt_lens = tgt_lens.int()
        loss, alpha, log_P_blank, log_P_y, log_prob, stash = torch.ops.asr.rnnt_forward_stash(
            encoder.contiguous(), decoder.contiguous(), joint_W.contiguous(), targets, in_lens, tgt_lens, blank_idx,
            tf32, _lib.logit_stash_budget(),
        )
        ctx.save_for_backward(encoder, decoder, joint_W, targets, in_lens, tgt_lens, alpha, log_P_blank, log_P_y,
                              log_prob, stash)
        ctx.blank_idx = blank_idx
        ctx.tf32 = tf32
        return loss

    @staticmethod
    def backward(ctx, *grad_outputs):
        (grad_loss,) = grad_outputs
        enc, dec, W, targets, in_lens, tgt_lens, alpha, log_P_blank, log_P_y, log_prob, stash = ctx.saved_tensors
        grad_encoder, grad_decoder, grad_joint_W = torch.ops.asr.rnnt_backward_stash(
            enc.contiguous(), dec.contiguous(), W.contiguous(), targets, in_lens, tgt_lens, ctx.blank_idx, alpha,
            log_P_blank, log_P_y, log_prob, grad_loss.contiguous(), ctx.tf32, stash,
        )
        return grad_encoder, grad_decoder, grad_joint_W, None, None, None, None, None


def rnnt_loss(encoder, decoder, joint_W, targets, in_lens, tgt_lens, blank_idx: int = 0, tf32: bool = False):
    """Per-utterance RNN-T loss ``-log P(y|x)`` (CUDA tensors; encoder / decoder
    float32, or bfloat16 to pass a system's autocast activations without float32
    copies: their gradients then come back in bfloat16).

    encoder (B, T, d), decoder (B, U, d) with U = max target length + 1 (the
    caller prepends <sos>), joint_W (V, d), targets (B, S >= U-1),
    in_lens (B,) in [1, T], tgt_lens (B,) in [0, U-1].
    """
    return RNNTLossFn.apply(encoder, decoder, joint_W, in_lens, tgt_lens, targets, blank_idx, int(tf32))


class RNNTLoss(torch.nn.Module):
    """RNN-T loss normalised per utterance by ``tgt_lens.clamp_min(1)``.

    Args:
        blank_idx: vocabulary index of the blank symbol.
        tf32: use the bf16 tensor-core joint network (fp32 accumulation).
    """

    def __init__(self, blank_idx: int = 0, tf32: bool = False):
        super().__init__()
        self.blank_idx = blank_idx
        self.tf32 = tf32

    def forward(self, encoder, decoder, joint_W, targets, in_lens, tgt_lens):
        loss = rnnt_loss(encoder, decoder, joint_W, targets, in_lens, tgt_lens, self.blank_idx, self.tf32)
        return loss / tgt_lens.clamp_min(1)


@dataclass
class RNNTLossConfig:
    _target_: str = "asr_b200.loss.rnnt.RNNTLoss"
    blank_idx: int = 0
    tf32: bool = False
