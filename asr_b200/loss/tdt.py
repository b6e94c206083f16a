"""TDT loss on the B200 kernels (interface of reference src/asr/loss/tdt.py:12-215)."""

from collections.abc import Sequence
from dataclasses import dataclass

import torch

from asr_b200 import _lib

_lib.load_ops()

# Device copies of duration lists, so repeated calls do not re-upload them.
_durations_cache: dict[tuple, torch.Tensor] = {}


def _durations_tensor(durations: list[int], device) -> torch.Tensor:
    key = (tuple(durations), str(device))
    t = _durations_cache.get(key)
    if t is None:
        t = torch.as_tensor(durations, dtype=torch.int32, device=device)
        _durations_cache[key] = t
    return t


class TDTLossFn(torch.autograd.Function):
    """Fused two-head joint network + Token-and-Duration Transducer loss.

    The forward keeps the joint's logits in a stash of at most
    ``asr_b200._lib.logit_stash_budget()`` bytes until the backward, which then
    forms d loss / d logits from it instead of recomputing the logits GEMM.
    """

    @staticmethod
    def forward(ctx, encoder, decoder, joint_W, joint_W_dur, in_lens, tgt_lens, targets, durations, max_duration,
                has_zero, blank_idx, sigma, tf32):
        targets = targets.int()
        in_lens = in_lens.int()
        tgt_lens = tgt_lens.int()
        durations = durations.int()
        loss, alpha, log_P_blank, log_P_y, log_P_dur, log_prob, stash = torch.ops.asr.tdt_forward_stash(
            encoder.contiguous(), decoder.contiguous(), joint_W.contiguous(), joint_W_dur.contiguous(), targets,
            in_lens, tgt_lens, durations, max_duration, has_zero, blank_idx, sigma, tf32, _lib.logit_stash_budget(),
        )
        ctx.save_for_backward(encoder, decoder, joint_W, joint_W_dur, targets, in_lens, tgt_lens, durations, alpha,
                              log_P_blank, log_P_y, log_P_dur, log_prob, stash)
        ctx.max_duration = max_duration
        ctx.has_zero = has_zero
        ctx.blank_idx = blank_idx
        ctx.tf32 = tf32
        return loss

    @staticmethod
    def backward(ctx, *grad_outputs):
        (grad_loss,) = grad_outputs
        (enc, dec, W, W_dur, targets, in_lens, tgt_lens, durations, alpha, log_P_blank, log_P_y, log_P_dur,
         log_prob, stash) = ctx.saved_tensors
        grad_encoder, grad_decoder, grad_joint_W, grad_joint_W_dur = torch.ops.asr.tdt_backward_stash(
            enc.contiguous(), dec.contiguous(), W.contiguous(), W_dur.contiguous(), targets, in_lens, tgt_lens,
            durations, ctx.max_duration, ctx.has_zero, ctx.blank_idx, alpha, log_P_blank, log_P_y, log_P_dur,
            log_prob, grad_loss.contiguous(), ctx.tf32, stash,
        )
        return (grad_encoder, grad_decoder, grad_joint_W, grad_joint_W_dur) + (None,) * 9


def tdt_loss(encoder, decoder, joint_W, joint_W_dur, targets, in_lens, tgt_lens, durations: Sequence[int],
             blank_idx: int = 0, sigma: float = 0.0, tf32: bool = False):
    """Per-utterance TDT loss ``-log P(y|x)`` with exact landing at (in_lens, tgt_lens).

    ``durations`` lists the frame advance of each joint_W_dur row; it must be
    non-negative and contain 1. ``sigma`` (>= 0) is the logit under-normalisation
    subtracted from every token log-prob (Xu et al. 2023, sec. 3.3). encoder /
    decoder may be float32 or bfloat16 (a system's autocast activations, passed
    without float32 copies; their gradients then come back in bfloat16); the
    joint weights stay float32.
    """
    durations = list(durations)
    if len(durations) != joint_W_dur.shape[0]:
        raise ValueError(f"len(durations)={len(durations)} must equal joint_W_dur rows={joint_W_dur.shape[0]}")
    if min(durations) < 0:
        raise ValueError(f"durations must be non-negative, got {durations}")
    if 1 not in durations:
        raise ValueError(f"durations must contain 1 so every frame count is reachable, got {durations}")
    if sigma < 0:
        raise ValueError(f"sigma must be non-negative, got {sigma}")
    durations_t = _durations_tensor(durations, encoder.device)
    return TDTLossFn.apply(encoder, decoder, joint_W, joint_W_dur, in_lens, tgt_lens, targets, durations_t,
                           int(max(durations)), int(0 in durations), blank_idx, float(sigma), int(tf32))


class TDTLoss(torch.nn.Module):
    """TDT loss normalised per utterance by ``tgt_lens.clamp_min(1)``.

    Args:
        max_duration: largest frame skip; durations are ``range(max_duration + 1)``.
        blank_idx: vocabulary index of the blank symbol.
        sigma: token logit under-normalisation offset.
        tf32: use the bf16 tensor-core joint network (fp32 accumulation).
    """

    def __init__(self, max_duration: int = 4, blank_idx: int = 0, sigma: float = 0.0, tf32: bool = False):
        super().__init__()
        if max_duration < 1:
            raise ValueError(f"max_duration must be >= 1, got {max_duration}")
        self.max_duration = max_duration
        self.durations = list(range(max_duration + 1))
        self.blank_idx = blank_idx
        self.sigma = sigma
        self.tf32 = tf32

    def forward(self, encoder, decoder, joint_W, joint_W_dur, targets, in_lens, tgt_lens):
        loss = tdt_loss(encoder, decoder, joint_W, joint_W_dur, targets, in_lens, tgt_lens, self.durations,
                        self.blank_idx, self.sigma, self.tf32)
        return loss / tgt_lens.clamp_min(1)


@dataclass
class TDTLossConfig:
    _target_: str = "asr_b200.loss.tdt.TDTLoss"
    max_duration: int = 4
    blank_idx: int = 0
    sigma: float = 0.0
    tf32: bool = False
