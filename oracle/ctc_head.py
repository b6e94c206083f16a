"""TEST INFRASTRUCTURE ONLY: float64 restatement of the reference CTC system's head
and loss, the checker for asr_b200.loss.ctc_head. Nothing in the product imports it.

Follows src/asr/system/ctc.py:21-24 and :36-40 (Sequential(RMSNorm(d), Linear(d, V))
under bf16 autocast, then CTCLoss) and src/asr/loss/ctc.py:11-30 (fp32
log_softmax, the CTC recursion, zero_infinity):
  * RMSNorm as torch computes it for a float32 input: x * rsqrt(mean(x^2) + eps) * g
    in float32 (eps = float32 epsilon by default);
  * the autocast Linear's operands rounded to bfloat16 (its input, weight and bias),
    products and sums in float64;
  * log_softmax and the CTC loss / gradient by the C oracle (oracle.ctc), then the
    chain rule back through the Linear and the RMSNorm in float64 (the bf16
    roundings pass gradients through unchanged, as autograd's casts do).
"""

from __future__ import annotations

import numpy as np

from oracle import oracle


def bf16(x):
    """Round float32 values to bfloat16 (nearest, ties to even); returns float64."""
    a = np.ascontiguousarray(np.asarray(x, np.float32))
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32).astype(np.float64)


def ctc_head(enc, g, W, b, targets, in_lens, tgt_lens, eps=np.finfo(np.float32).eps, zero_infinity=False,
             grad_loss=None):
    x = np.asarray(enc, np.float32)
    B, T, d = x.shape
    ms = np.mean(x.astype(np.float32) ** 2, axis=-1, keepdims=True, dtype=np.float32)
    rstd = (1.0 / np.sqrt(ms + np.float32(eps))).astype(np.float32)
    y = (x * rstd * np.asarray(g, np.float32)).astype(np.float32)
    h = bf16(y)
    Wb = bf16(W)
    bb = bf16(b) if b is not None else np.zeros(W.shape[0])
    logits = h @ Wb.T + bb
    m = logits.max(-1, keepdims=True)
    lp = logits - (m + np.log(np.exp(logits - m).sum(-1, keepdims=True)))
    gl = np.ones(B, np.float32) if grad_loss is None else np.asarray(grad_loss, np.float32)
    loss, G = oracle.ctc(lp.astype(np.float32), targets, in_lens, tgt_lens, grad_loss=gl,
                         zero_infinity=zero_infinity)
    if zero_infinity:
        loss = np.where(np.isfinite(loss), loss, 0.0)
    out = {"loss": loss}
    dW = np.einsum("btv,btk->vk", G, h)
    out["dW"] = dW
    if b is not None:
        out["db"] = G.sum((0, 1))
    dy = G @ Wb                                   # d loss / d RMSNorm output
    xh = x.astype(np.float64) * rstd
    gg = np.asarray(g, np.float64)
    out["dg"] = (dy * xh).sum((0, 1))
    c = (xh * gg * dy).mean(-1, keepdims=True)
    out["d_enc"] = rstd * (gg * dy - xh * c)
    return out
