"""Fused CTC head + loss: the reference CTC system's ``Linear(RMSNorm(enc))`` head
(src/asr/system/ctc.py:21-24) and ``CTCLoss`` (src/asr/loss/ctc.py:11-63) in one op
whose (B, T, V) logits, log-probs and logit gradients never reach HBM.

``FusedCTCHead`` is the head module itself (a ``torch.nn.Sequential(RMSNorm,
Linear)``, so its state dict matches the reference's ``system.head``) with a
second calling form that returns the loss:

    head = FusedCTCHead(d_model, n_vocab, zero_infinity=True)
    logits = head(enc)                                   # the plain head, for decoding
    loss = head(enc, targets, in_lens, tgt_lens)         # fused: CTCLoss(head(enc), ...)

The fused form runs the GEMM as bf16 tcgen05 tensor-core MMAs with fp32
accumulation on bf16(RMSNorm(enc)) and bf16(weight, bias), the operands the
reference's bf16-autocast Linear uses.
"""

from __future__ import annotations

import ctypes

import torch

from asr_b200 import _lib

_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float
_bound = False


def _capi() -> ctypes.CDLL:
    global _bound
    lib = _lib.capi()
    if not _bound:
        lib.asr_ctc_head_workspace_bytes.restype = ctypes.c_size_t
        lib.asr_ctc_head_workspace_bytes.argtypes = [_I] * 6
        lib.asr_ctc_head_supported.argtypes = [_I, _I]
        lib.asr_ctc_head_forward.argtypes = [_P, _I, _P, _F, _P, _P, _P, _P, _P] + [_I] * 6 + [_P, _P, ctypes.c_size_t,
                                                                                            _P]
        lib.asr_ctc_head_backward.argtypes = [_P, _I, _P, _F, _P, _P, _P, _P, _P] + [_I] * 6 + [_P] * 6 + [
            ctypes.c_size_t, _P]
        lib.asr_status_string.restype = ctypes.c_char_p
        _bound = True
    return lib


def _check(lib, rc, what):
    if rc != 0:
        raise RuntimeError(f"{what} failed: {lib.asr_status_string(rc).decode()} (status {rc})")


def _ptr(t):
    return None if t is None else t.data_ptr()


class CTCHeadLossFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, enc, rms_weight, weight, bias, targets, in_lens, tgt_lens, eps, zero_infinity):
        if not enc.is_cuda:
            raise RuntimeError("the fused CTC head runs on CUDA tensors only (there is no CPU path)")
        if enc.dtype not in (torch.float32, torch.bfloat16):
            raise TypeError(f"encoder output must be float32 or bfloat16, got {enc.dtype}")
        enc = enc.contiguous()
        rms_weight = rms_weight.detach().float().contiguous()
        weight = weight.detach().float().contiguous()
        bias = None if bias is None else bias.detach().float().contiguous()
        targets = targets.int().contiguous()
        in_lens = in_lens.int().contiguous()
        tgt_lens = tgt_lens.int().contiguous()
        B, T, d = enc.shape
        V = weight.shape[0]
        S = targets.shape[1] if targets.dim() == 2 else 0
        act = 1 if enc.dtype == torch.bfloat16 else 0
        lib = _capi()
        nbytes = lib.asr_ctc_head_workspace_bytes(B, T, S, V, d, act)
        ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=enc.device)
        loss = torch.empty(B, dtype=torch.float32, device=enc.device)
        stream = ctypes.c_void_p(torch.cuda.current_stream(enc.device).cuda_stream)
        _check(lib, lib.asr_ctc_head_forward(
            enc.data_ptr(), act, rms_weight.data_ptr(), float(eps), weight.data_ptr(), _ptr(bias),
            _ptr(targets) if S else None, in_lens.data_ptr(), tgt_lens.data_ptr(), B, T, S, V, d,
            int(bool(zero_infinity)), loss.data_ptr(), ws.data_ptr(), nbytes, stream), "asr_ctc_head_forward")
        ctx.save_for_backward(enc, rms_weight, weight, bias, targets, in_lens, tgt_lens)
        ctx.ws = ws
        ctx.eps = float(eps)
        ctx.zero_infinity = int(bool(zero_infinity))
        ctx.has_bias = bias is not None
        return loss

    @staticmethod
    def backward(ctx, grad_loss):
        enc, rms_weight, weight, bias, targets, in_lens, tgt_lens = ctx.saved_tensors
        B, T, d = enc.shape
        V = weight.shape[0]
        S = targets.shape[1] if targets.dim() == 2 else 0
        act = 1 if enc.dtype == torch.bfloat16 else 0
        grad_loss = grad_loss.float().contiguous()
        d_enc = torch.empty_like(enc)
        d_g = torch.empty(d, dtype=torch.float32, device=enc.device)
        d_W = torch.empty(V, d, dtype=torch.float32, device=enc.device)
        d_b = torch.empty(V, dtype=torch.float32, device=enc.device) if ctx.has_bias else None
        lib = _capi()
        stream = ctypes.c_void_p(torch.cuda.current_stream(enc.device).cuda_stream)
        _check(lib, lib.asr_ctc_head_backward(
            enc.data_ptr(), act, rms_weight.data_ptr(), ctx.eps, weight.data_ptr(), _ptr(bias),
            _ptr(targets) if S else None, in_lens.data_ptr(), tgt_lens.data_ptr(), B, T, S, V, d, ctx.zero_infinity,
            grad_loss.data_ptr(), d_enc.data_ptr(), d_g.data_ptr(), d_W.data_ptr(), _ptr(d_b), ctx.ws.data_ptr(),
            ctx.ws.numel(), stream), "asr_ctc_head_backward")
        ctx.ws = None
        return d_enc, d_g, d_W, d_b, None, None, None, None, None


def ctc_head_loss(enc, rms_weight, weight, bias, targets, in_lens, tgt_lens, eps=None, zero_infinity=False):
    """Per-utterance ``-log P(targets | enc)`` of ``log_softmax(Linear(RMSNorm(enc)))``
    (blank = 0), not normalised by the target lengths. ``eps=None`` is torch's
    RMSNorm default (float32 epsilon)."""
    if eps is None:
        eps = torch.finfo(torch.float32).eps
    return CTCHeadLossFn.apply(enc, rms_weight, weight, bias, targets, in_lens, tgt_lens, eps, zero_infinity)


class FusedCTCHead(torch.nn.Sequential):
    """``Sequential(RMSNorm(d_model), Linear(d_model, n_vocab))`` whose 4-argument
    call fuses the head with ``CTCLoss`` (divided by ``tgt_lens.clamp_min(1)`` as
    the reference module divides)."""

    def __init__(self, d_model: int, n_vocab: int, zero_infinity: bool = False, eps: float | None = None,
                 bias: bool = True):
        super().__init__(torch.nn.RMSNorm(d_model, eps=eps), torch.nn.Linear(d_model, n_vocab, bias=bias))
        self.zero_infinity = zero_infinity

    def forward(self, enc, targets=None, in_lens=None, tgt_lens=None):
        if targets is None:
            return super().forward(enc)
        norm, lin = self[0], self[1]
        loss = ctc_head_loss(enc, norm.weight, lin.weight, lin.bias, targets, in_lens, tgt_lens, norm.eps,
                             self.zero_infinity)
        return loss / tgt_lens.clamp_min(1)
