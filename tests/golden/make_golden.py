"""Generate the golden parity fixtures under ``tests/golden/`` from the reference itself.

Run once in a container that has the reference checkout (it imports the
reference's own float64 oracles, which are not shipped with this repo):

    python tests/golden/make_golden.py --reference /path/to/samgd-asr

Inputs are drawn from seeded numpy generators and rounded to float32 (what the
CUDA path consumes); the expected losses and gradients are computed from those
float32 values in float64 by
  - CTC   : ``torch.nn.functional.ctc_loss`` (the oracle of tests/loss/test_ctc_loss.py:49-58),
  - RNN-T : ``tests/loss/rnnt_reference.py`` (rnnt_loss, analytic backward),
  - TDT   : ``tests/loss/tdt_reference.py`` (tdt_loss, analytic backward),
so the fixtures pin both the C oracle and the CUDA kernels to the reference.
The case list covers the edge cases the reference's tests exercise: padding,
empty targets, all-empty batches, repeated CTC labels, weighted upstream grads,
several max durations and sigma values.
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _lengths(rng, B, lo, hi):
    return rng.integers(lo, hi + 1, size=B).astype(np.int32)


def ctc_cases():
    # (name, B, T, V, S, in_lens, tgt_lens, seed, zero_infinity, weights)
    yield "trivial", 1, 4, 3, 1, None, None, 0, False, None
    yield "tight_T_eq_2S+1", 1, 5, 4, 2, None, None, 1, False, None
    yield "small_fixed", 4, 20, 8, 6, None, None, 2, False, None
    yield "varlen_padded", 3, 30, 10, 8, [30, 25, 20], [8, 5, 3], 3, False, None
    yield "larger_fixed", 8, 50, 29, 20, None, None, 4, False, None
    yield "empty_target", 2, 10, 5, 3, [10, 7], [3, 0], 5, False, None
    yield "weighted", 3, 15, 6, 4, None, None, 6, False, [0.5, 2.0, 1.5]
    yield "repeats", 1, 6, 5, 3, [6], [3], 7, False, None  # labels forced to [1,1,2]
    yield "infeasible_zero_inf", 2, 4, 5, 3, [4, 4], [3, 1], 8, True, None
    yield "config1_like", 8, 200, 29, 60, "cfg1", "cfg1", 9, False, None


def make_ctc(out):
    import torch.nn.functional as F

    for name, B, T, V, S, il, tl, seed, zinf, w in ctc_cases():
        rng = np.random.default_rng(1000 + seed)
        logits = rng.standard_normal((B, T, V)).astype(np.float32)
        targets = rng.integers(1, V, size=(B, S)).astype(np.int32)
        if name == "repeats":
            targets[0, :3] = [1, 1, 2]
        if il == "cfg1":
            il = _lengths(rng, B, 150, 200)
            tl = _lengths(rng, B, 20, 60)
        in_lens = np.full(B, T, np.int32) if il is None else np.asarray(il, np.int32)
        tgt_lens = np.full(B, S, np.int32) if tl is None else np.asarray(tl, np.int32)
        weights = np.ones(B, np.float32) if w is None else np.asarray(w, np.float32)
        x = torch.tensor(logits, dtype=torch.float64, requires_grad=True)
        lp = x.log_softmax(-1)
        loss = F.ctc_loss(lp.transpose(0, 1), torch.tensor(targets).long(), torch.tensor(in_lens).long(),
                          torch.tensor(tgt_lens).long(), blank=0, reduction="none", zero_infinity=zinf)
        (loss * torch.tensor(weights, dtype=torch.float64)).sum().backward()
        out[f"ctc/{name}/logits"] = logits
        out[f"ctc/{name}/log_probs"] = torch.tensor(logits).log_softmax(-1).numpy()
        out[f"ctc/{name}/targets"] = targets
        out[f"ctc/{name}/in_lens"] = in_lens
        out[f"ctc/{name}/tgt_lens"] = tgt_lens
        out[f"ctc/{name}/grad_loss"] = weights
        out[f"ctc/{name}/zero_infinity"] = np.array(int(zinf))
        out[f"ctc/{name}/loss"] = loss.detach().numpy()
        out[f"ctc/{name}/grad_logits"] = x.grad.numpy()


def transducer_cases():
    # (name, B, T, U, V, d, in_lens, tgt_lens, seed, weights)
    yield "single", 1, 4, 3, 5, 6, None, None, 0, None
    yield "batch_fixed", 4, 12, 6, 8, 8, None, None, 1, None
    yield "variable_lens", 3, 15, 6, 10, 8, [15, 12, 9], [5, 3, 1], 2, None
    yield "empty_target_in_batch", 2, 5, 3, 4, 4, [5, 4], [2, 0], 3, None
    yield "all_empty_targets", 2, 4, 1, 4, 3, None, None, 4, None
    yield "padding", 2, 6, 4, 5, 4, [6, 4], [3, 1], 5, None
    yield "weighted", 3, 8, 5, 6, 6, None, None, 6, [0.5, 2.0, 1.5]
    yield "wider", 2, 20, 9, 33, 40, [20, 17], [8, 5], 7, None


def _transducer_inputs(rng, B, T, U, V, d, n_dur=0, scale=1.0):
    enc = (rng.standard_normal((B, T, d)) * scale).astype(np.float32)
    dec = (rng.standard_normal((B, U, d)) * scale).astype(np.float32)
    W = rng.standard_normal((V, d)).astype(np.float32)
    Wd = rng.standard_normal((n_dur, d)).astype(np.float32) if n_dur else None
    targets = rng.integers(1, V, size=(B, max(U - 1, 0))).astype(np.int32)
    return enc, dec, W, Wd, targets


def make_rnnt(out, ref):
    from tests.loss.rnnt_reference import rnnt_loss as rnnt_ref

    for name, B, T, U, V, d, il, tl, seed, w in transducer_cases():
        rng = np.random.default_rng(2000 + seed)
        enc, dec, W, _, targets = _transducer_inputs(rng, B, T, U, V, d)
        in_lens = np.full(B, T, np.int32) if il is None else np.asarray(il, np.int32)
        tgt_lens = np.full(B, U - 1, np.int32) if tl is None else np.asarray(tl, np.int32)
        weights = np.ones(B, np.float32) if w is None else np.asarray(w, np.float32)
        e, dd, ww = (torch.tensor(a, dtype=torch.float64, requires_grad=True) for a in (enc, dec, W))
        loss = rnnt_ref(e, dd, ww, torch.tensor(targets), torch.tensor(in_lens), torch.tensor(tgt_lens), 0)
        (loss * torch.tensor(weights, dtype=torch.float64)).sum().backward()
        p = f"rnnt/{name}/"
        out[p + "enc"], out[p + "dec"], out[p + "W"], out[p + "targets"] = enc, dec, W, targets
        out[p + "in_lens"], out[p + "tgt_lens"], out[p + "grad_loss"] = in_lens, tgt_lens, weights
        out[p + "loss"] = loss.detach().numpy()
        out[p + "d_enc"], out[p + "d_dec"], out[p + "dW"] = e.grad.numpy(), dd.grad.numpy(), ww.grad.numpy()


def tdt_cases():
    # (name, B, T, U, V, d, max_duration, in_lens, tgt_lens, seed, sigma, weights)
    yield "single", 1, 4, 3, 5, 6, 4, None, None, 0, 0.0, None
    yield "batch_fixed_s005", 4, 12, 6, 8, 8, 4, None, None, 1, 0.05, None
    yield "variable_lens_s02", 3, 15, 6, 10, 8, 4, [15, 12, 9], [5, 3, 1], 2, 0.2, None
    yield "empty_target_in_batch", 2, 5, 3, 4, 4, 2, [5, 4], [2, 0], 3, 0.0, None
    yield "max_duration_2", 4, 12, 6, 8, 8, 2, None, None, 4, 0.05, None
    yield "max_duration_6", 3, 12, 5, 6, 6, 6, [12, 10, 8], [4, 3, 2], 5, 0.0, None
    yield "max_duration_1", 2, 7, 4, 6, 5, 1, [7, 5], [3, 2], 6, 0.1, None
    yield "weighted", 3, 8, 5, 6, 6, 3, None, None, 7, 0.0, [0.5, 2.0, 1.5]
    yield "padding", 2, 6, 4, 5, 4, 2, [6, 4], [3, 1], 8, 0.0, None
    yield "all_empty_targets", 2, 5, 1, 4, 3, 3, None, None, 9, 0.05, None
    yield "wider", 2, 20, 9, 33, 40, 4, [20, 17], [8, 5], 10, 0.05, None


def make_tdt(out, ref):
    from tests.loss.tdt_reference import tdt_loss as tdt_ref

    for name, B, T, U, V, d, md, il, tl, seed, sigma, w in tdt_cases():
        rng = np.random.default_rng(3000 + seed)
        durations = list(range(md + 1))
        enc, dec, W, Wd, targets = _transducer_inputs(rng, B, T, U, V, d, n_dur=len(durations))
        in_lens = np.full(B, T, np.int32) if il is None else np.asarray(il, np.int32)
        tgt_lens = np.full(B, U - 1, np.int32) if tl is None else np.asarray(tl, np.int32)
        weights = np.ones(B, np.float32) if w is None else np.asarray(w, np.float32)
        e, dd, ww, wd = (torch.tensor(a, dtype=torch.float64, requires_grad=True) for a in (enc, dec, W, Wd))
        loss = tdt_ref(e, dd, ww, wd, torch.tensor(targets), torch.tensor(in_lens), torch.tensor(tgt_lens), durations,
                       0, sigma)
        (loss * torch.tensor(weights, dtype=torch.float64)).sum().backward()
        p = f"tdt/{name}/"
        out[p + "enc"], out[p + "dec"], out[p + "W"], out[p + "W_dur"] = enc, dec, W, Wd
        out[p + "targets"], out[p + "in_lens"], out[p + "tgt_lens"] = targets, in_lens, tgt_lens
        out[p + "durations"] = np.asarray(durations, np.int32)
        out[p + "sigma"] = np.array(sigma, np.float64)
        out[p + "grad_loss"] = weights
        out[p + "loss"] = loss.detach().numpy()
        out[p + "d_enc"], out[p + "d_dec"] = e.grad.numpy(), dd.grad.numpy()
        out[p + "dW"], out[p + "dW_dur"] = ww.grad.numpy(), wd.grad.numpy()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="checkout of the reference repository (read-only)")
    args = ap.parse_args()
    sys.path.insert(0, str(Path(args.reference)))
    torch.set_default_dtype(torch.float64)
    for kind, fn in (("ctc", make_ctc), ("rnnt", make_rnnt), ("tdt", make_tdt)):
        out: dict[str, np.ndarray] = {}
        fn(out) if kind == "ctc" else fn(out, args.reference)
        np.savez_compressed(HERE / f"{kind}_golden.npz", **out)
        print(kind, len(out), "arrays")


if __name__ == "__main__":
    main()
