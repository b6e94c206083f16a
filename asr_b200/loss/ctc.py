"""CTC loss on the B200 kernels (interface of reference src/asr/loss/ctc.py:11-69)."""

from dataclasses import dataclass

import torch

from asr_b200 import _lib

_lib.load_ops()


class CTCLossFn(torch.autograd.Function):
    """Per-utterance CTC loss ``-log Z`` with the fused beta/gradient backward.

    Forward normalises ``logits`` with a float32 log-softmax, then runs the
    alpha recursion (``asr::ctc_alpha``); backward returns d loss / d logits
    (``asr::ctc_grad``), already pushed through the log-softmax.
    """

    @staticmethod
    def forward(ctx, logits, targets, in_lens, tgt_lens, zero_infinity):
        log_probs = torch.nn.functional.log_softmax(logits.float(), dim=-1)
        alpha, log_Z = torch.ops.asr.ctc_alpha(log_probs, targets, in_lens, tgt_lens)
        ctx.save_for_backward(log_probs, alpha, log_Z, targets, in_lens, tgt_lens)
        ctx.zero_infinity = zero_infinity
        loss = -log_Z
        if zero_infinity:
            loss = torch.where(torch.isfinite(loss), loss, torch.zeros_like(loss))
        return loss

    @staticmethod
    def backward(ctx, *grad_outputs):
        (grad_loss,) = grad_outputs
        log_probs, alpha, log_Z, targets, in_lens, tgt_lens = ctx.saved_tensors
        grad_logits = torch.ops.asr.ctc_grad(
            alpha, log_Z, log_probs, targets, in_lens, tgt_lens, grad_loss.contiguous(), ctx.zero_infinity
        )
        return grad_logits, None, None, None, None


class CTCLoss(torch.nn.Module):
    """Connectionist Temporal Classification loss, normalised by target length.

    Args:
        zero_infinity: replace infinite (infeasible) losses and their gradients with 0.

    Shape:
        x: (B, T, V) logits (log-softmax is applied inside), blank at index 0.
        targets: (B, S_max) label ids; in_lens: (B,) in [1, T]; tgt_lens: (B,) in [0, S_max].
    """

    def __init__(self, zero_infinity: bool = False):
        super().__init__()
        self.zero_infinity = zero_infinity

    def forward(self, x, targets, in_lens, tgt_lens):
        loss = CTCLossFn.apply(x, targets.int(), in_lens.int(), tgt_lens.int(), self.zero_infinity)
        return loss / tgt_lens.clamp_min(1)


@dataclass
class CTCLossConfig:
    _target_: str = "asr_b200.loss.ctc.CTCLoss"
    zero_infinity: bool = False
