"""Generate ``tests/golden/ctc_head_golden.npz``: losses and gradients of the reference
CTC system's head and loss, computed by torch in float64.

The reference path (src/asr/system/ctc.py:21-24 and :36-40, src/asr/loss/ctc.py:11-30)
is ``CTCLoss(Linear(RMSNorm(enc)))`` under bf16 autocast. This script builds exactly
that head with ``torch.nn.RMSNorm`` / ``torch.nn.Linear``:
  * RMSNorm runs in float32 (autocast's float32 op; eps = float32 epsilon);
  * the Linear's input, weight and bias are rounded to bfloat16 as autocast does,
    and the product is then taken in float64 (straight-through: the roundings pass
    gradients unchanged, as autograd's casts do, so the expected gradients are
    exact for the rounded operands);
  * the loss is ``torch.nn.functional.ctc_loss`` in float64, the oracle the
    reference's own CTC tests use (tests/loss/test_ctc_loss.py:49-58), blank = 0,
    reduction "none", with the reference's zero_infinity option.
It needs no reference checkout: the reference CTC loss itself requires its CUDA
extension, and its tests pin it to ``F.ctc_loss``.

    python tests/golden/make_ctc_head_golden.py
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def st_bf16(x):
    return x + (x.to(torch.bfloat16).to(x.dtype) - x).detach()


def cases():
    # (name, B, T, d, V, S, in_lens, tgt_lens, bias, zero_infinity, weights, seed)
    yield "tiny", 1, 6, 16, 5, 2, [6], [2], True, False, None, 0
    yield "small", 3, 20, 32, 12, 6, [20, 15, 9], [6, 4, 2], True, False, None, 1
    yield "no_bias", 2, 16, 24, 10, 5, [16, 12], [5, 3], False, False, None, 2
    yield "repeats", 2, 18, 32, 8, 6, [18, 18], [6, 6], True, False, None, 3  # labels forced to repeat
    yield "empty_target", 2, 10, 16, 6, 3, [10, 7], [3, 0], True, False, None, 4
    yield "weighted", 3, 14, 32, 9, 4, [14, 11, 8], [4, 4, 2], True, False, [0.5, 2.0, 1.5], 5
    yield "infeasible_zero_inf", 2, 4, 16, 6, 3, [4, 4], [3, 1], True, True, None, 6
    yield "odd_dims", 3, 25, 67, 37, 7, [25, 20, 13], [7, 5, 2], True, False, None, 7
    yield "wide_vocab", 2, 30, 64, 300, 10, [30, 24], [10, 8], True, False, None, 8
    yield "config1_like", 8, 200, 64, 29, 60, "cfg1", "cfg1", True, True, None, 9


def make(out):
    for name, B, T, d, V, S, il, tl, has_bias, zinf, w, seed in cases():
        rng = np.random.default_rng(3000 + seed)
        if il == "cfg1":
            il = rng.integers(150, T + 1, size=B)
            tl = rng.integers(20, S + 1, size=B)
        il = np.asarray(il, np.int32)
        tl = np.asarray(tl, np.int32)
        enc = rng.standard_normal((B, T, d)).astype(np.float32)
        g = (1.0 + 0.1 * rng.standard_normal(d)).astype(np.float32)
        W = (rng.standard_normal((V, d)) / np.sqrt(d)).astype(np.float32)
        bias = (0.1 * rng.standard_normal(V)).astype(np.float32) if has_bias else None
        targets = rng.integers(1, V, size=(B, S)).astype(np.int32)
        if name == "repeats":
            targets[0, :6] = [3, 3, 5, 5, 5, 2]
            targets[1, :6] = [1, 2, 1, 2, 1, 2]
        if name == "infeasible_zero_inf":
            targets[0, :3] = [2, 2, 2]  # needs 5 frames, has 4: -log P = inf, dropped
        weights = np.asarray(w if w is not None else np.ones(B), np.float32)

        e = torch.tensor(enc, dtype=torch.float32, requires_grad=True)
        norm = torch.nn.RMSNorm(d)
        with torch.no_grad():
            norm.weight.copy_(torch.from_numpy(g))
        y = norm(e)                                   # float32, as under autocast
        gW = torch.tensor(W, dtype=torch.float64, requires_grad=True)
        gb = torch.tensor(bias, dtype=torch.float64, requires_grad=True) if has_bias else None
        logits = st_bf16(y.double()) @ st_bf16(gW).T
        if has_bias:
            logits = logits + st_bf16(gb)
        lp = torch.log_softmax(logits, -1)
        loss = torch.nn.functional.ctc_loss(lp.transpose(0, 1), torch.from_numpy(targets).long(),
                                            torch.from_numpy(il).long(), torch.from_numpy(tl).long(), blank=0,
                                            reduction="none", zero_infinity=zinf)
        (loss * torch.from_numpy(weights).double()).sum().backward()
        p = f"ctc_head/{name}/"
        out[p + "enc"], out[p + "g"], out[p + "W"] = enc, g, W
        if has_bias:
            out[p + "b"] = bias
        out[p + "targets"], out[p + "in_lens"], out[p + "tgt_lens"] = targets, il, tl
        out[p + "zero_infinity"] = np.array(int(zinf), np.int32)
        out[p + "grad_loss"] = weights
        out[p + "loss"] = loss.detach().numpy()
        # gradients stored in float32 (plenty for the 1e-6 oracle pin; halves the file)
        out[p + "d_enc"] = e.grad.float().numpy()
        out[p + "dg"] = norm.weight.grad.float().numpy()
        out[p + "dW"] = gW.grad.float().numpy()
        if has_bias:
            out[p + "db"] = gb.grad.float().numpy()
        print(name, "loss", np.round(loss.detach().numpy()[:3], 4))


def main():
    out: dict[str, np.ndarray] = {}
    make(out)
    np.savez_compressed(HERE / "ctc_head_golden.npz", **out)
    print("ctc_head", len(out), "arrays")


if __name__ == "__main__":
    main()
