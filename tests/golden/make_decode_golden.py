"""Generate ``tests/golden/decode_golden.npz`` from the reference's own greedy decoders.

Run once in a container that has the reference checkout (it imports
``src/asr/decode/rnnt.py`` and ``src/asr/decode/tdt.py`` from it; they need
torch and jaxtyping):

    python tests/golden/make_decode_golden.py --reference /path/to/samgd-asr

Every case runs the reference ``greedy_decode`` on CPU with
  * the systems' joint: ``Linear(W, bias=False)(tanh(enc_t + pred_u))``
    (src/asr/system/rnnt.py:29-34, src/asr/system/tdt.py:31-43), in float32;
  * a position-wise table predictor: ``predict(tokens)[..., i, :] =
    P[tokens[..., i]] + Q[(i + 1) % len(Q)]`` (float32), so the same values come
    out of any implementation of it.
Random cases are redrawn until every argmax the reference takes has a top-2
margin above 1e-3 (relative), so float32 rounding differences between
implementations cannot flip a decision; the stored ``min_margin`` records it.

The ``ref_*`` cases restate the scenarios of the reference's decoder tests
(tests/decode/test_tdt_decode.py): there the synthetic joint reads the
encoder vector directly; here W is the selection matrix [I_V | 0] (and
[0 | I_Dn] for durations) with a zero predictor, so argmax W tanh(enc) picks
the same entries.
"""

from __future__ import annotations

import argparse
import importlib.util
import sys
import zlib
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _load(ref: Path, name: str):
    spec = importlib.util.spec_from_file_location(f"ref_decode_{name}", ref / "src" / "asr" / "decode" / f"{name}.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.greedy_decode


class Margin:
    """Wraps a joint closure and records the smallest relative top-2 gap it returned."""

    def __init__(self, fn):
        self.fn = fn
        self.min = np.inf

    def __call__(self, e, p):
        z = self.fn(e, p)
        if z.numel() > 1:
            top = torch.topk(z, 2).values
            self.min = min(self.min, float((top[0] - top[1]) / max(1.0, abs(float(top[0])))))
        return z


def _joint(W):
    Wt = torch.from_numpy(W)
    return lambda e, p: torch.tanh(e + p) @ Wt.T


def _predictor(P, Q):
    Pt, Qt = torch.from_numpy(P), torch.from_numpy(Q)

    def predict(tokens):
        pos = (torch.arange(tokens.shape[-1]) + 1) % Qt.shape[0]
        return Pt[tokens] + Qt[pos]

    return predict


def random_case(rng, B, T, V, d, n_dur, lens):
    enc = (rng.standard_normal((B, T, d)) * 0.8).astype(np.float32)
    enc[..., 0] = 2.0  # a constant direction that W[blank] can weight
    W = (rng.standard_normal((V, d)) / np.sqrt(d) * 3.0).astype(np.float32)
    P = (rng.standard_normal((V, d)) * 0.5).astype(np.float32)
    Q = (rng.standard_normal((7, d)) * 0.3).astype(np.float32)
    c = dict(enc=enc, W=W, P=P, Q=Q, in_lens=np.asarray(lens, np.int32))
    if n_dur:
        c["W_dur"] = (rng.standard_normal((n_dur, d)) / np.sqrt(d) * 3.0).astype(np.float32)
    return c


def cases():
    # (name, kind, B, T, V, d, n_dur, blank, sos, max_sym, blank_bias, lens)
    yield "rnnt_small", "rnnt", 3, 12, 12, 16, 0, 0, 1, 10, 5.0, [12, 9, 5]
    yield "rnnt_max1", "rnnt", 2, 10, 12, 16, 0, 0, 1, 1, 0.0, [10, 7]
    yield "rnnt_cap3_no_blank", "rnnt", 2, 6, 10, 16, 0, 0, 1, 3, -4.0, [6, 4]
    yield "rnnt_zero_len", "rnnt", 3, 8, 12, 16, 0, 0, 1, 10, 5.0, [8, 0, 3]
    yield "rnnt_blank_last", "rnnt", 2, 14, 13, 24, 0, 12, 3, 4, 4.0, [14, 11]
    yield "rnnt_char30", "rnnt", 4, 40, 30, 40, 0, 0, 1, 10, 6.0, [40, 33, 21, 38]
    yield "rnnt_wide_vocab", "rnnt", 2, 20, 1100, 36, 0, 0, 1, 5, 8.0, [20, 13]
    yield "rnnt_odd_dim", "rnnt", 3, 25, 37, 67, 0, 0, 1, 10, 6.0, [25, 24, 10]
    yield "tdt_small", "tdt", 3, 16, 20, 32, 5, 0, 1, 10, 3.0, [16, 11, 6]
    yield "tdt_max1", "tdt", 2, 12, 20, 32, 3, 0, 1, 1, 0.5, [12, 8]
    yield "tdt_cap3_no_blank", "tdt", 2, 8, 12, 16, 3, 0, 1, 3, -4.0, [8, 5]
    yield "tdt_zero_len", "tdt", 3, 10, 16, 24, 5, 0, 1, 10, 1.0, [10, 0, 4]
    yield "tdt_blank_last", "tdt", 2, 18, 21, 24, 4, 20, 2, 6, 1.0, [18, 15]
    yield "tdt_bpe_like", "tdt", 4, 48, 96, 64, 5, 0, 1, 10, 5.0, [48, 40, 25, 31]
    yield "tdt_wide_vocab", "tdt", 2, 24, 1100, 36, 5, 0, 1, 5, 6.0, [24, 19]
    yield "tdt_odd_dim", "tdt", 3, 30, 37, 67, 5, 0, 1, 10, 1.5, [30, 22, 9]


def make_random(out, rnnt_dec, tdt_dec):
    for name, kind, B, T, V, d, n_dur, blank, sos, max_sym, bias, lens in cases():
        for attempt in range(200):
            rng = np.random.default_rng([zlib.crc32(name.encode()), attempt])
            c = random_case(rng, B, T, V, d, n_dur, lens)
            c["W"][blank, 0] += bias  # blank logit offset through the constant enc direction
            if n_dur:
                c["W_dur"][1, 0] += 0.5  # favour duration 1, as trained models do
            joint = Margin(_joint(c["W"]))
            predict = _predictor(c["P"], c["Q"])
            enc_t = torch.from_numpy(c["enc"])
            lens_t = torch.from_numpy(c["in_lens"])
            if kind == "rnnt":
                hyps = rnnt_dec(enc_t, lens_t, predict, joint, blank_id=blank, sos_id=sos,
                                max_symbols_per_frame=max_sym)
                durs = None
                margin = joint.min
            else:
                jd = Margin(_joint(c["W_dur"]))
                hyps, durs = tdt_dec(enc_t, lens_t, predict, joint, jd, n_dur - 1, blank_id=blank, sos_id=sos,
                                     max_symbols_per_frame=max_sym)
                margin = min(joint.min, jd.min)
            if margin > 1e-3:
                break
        else:
            raise RuntimeError(f"{name}: no draw with a safe argmax margin")
        _store(out, name, kind, c, blank, sos, max_sym, n_dur - 1 if n_dur else 0, hyps, durs, margin)
        print(f"{name}: attempt {attempt}, tokens {[len(h) for h in hyps]}, margin {margin:.2e}")


def _store(out, name, kind, c, blank, sos, max_sym, max_duration, hyps, durs, margin):
    p = f"decode/{name}/"
    for k, v in c.items():
        out[p + k] = v
    out[p + "kind"] = np.array(kind)
    out[p + "params"] = np.array([blank, sos, max_sym, max_duration], np.int32)
    out[p + "hyp_lens"] = np.array([len(h) for h in hyps], np.int32)
    out[p + "hyp_flat"] = np.array([x for h in hyps for x in h], np.int32)
    if durs is not None:
        out[p + "dur_lens"] = np.array([len(x) for x in durs], np.int32)
        out[p + "dur_flat"] = np.array([x for h in durs for x in h], np.int32)
    out[p + "min_margin"] = np.array(margin, np.float64)


def _plan_enc(plans, T, V, durations, default=(0, 1)):
    """(B, T, V + n_dur) frames whose selected (token, duration) entries are 10."""
    enc = np.zeros((len(plans), T, V + len(durations)), np.float32)
    for b, plan in enumerate(plans):
        for t in range(T):
            tok, dv = plan.get(t, default)
            enc[b, t, tok] = 10.0
            enc[b, t, V + durations.index(dv)] = 10.0
    return enc


def make_reference_scenarios(out, tdt_dec):
    # tests/decode/test_tdt_decode.py scenarios, as (name, plans, T, V, durations, in_lens, max_sym)
    scen = [
        ("ref_duration_one", [{t: (2, 1) for t in range(5)}], 5, 6, [0, 1, 2], [5], 10),
        ("ref_blank_duration_skips", [{t: (0, 2) for t in range(5)}], 5, 6, [0, 1, 2], [5], 10),
        ("ref_duration_zero_cap", [{t: (3, 0) for t in range(2)}], 2, 6, [0, 1, 2], [2], 3),
        ("ref_blank_zero_forces", [{t: (0, 0) for t in range(4)}], 4, 6, [0, 1, 2], [4], 10),
        ("ref_frame_skip", [{0: (2, 1), 1: (0, 2), 2: (9, 1), 3: (4, 1), 4: (0, 1), 5: (5, 3)}], 10, 10,
         [0, 1, 2, 3], [10], 10),
        ("ref_batch_in_lens", [{t: (2, 1) for t in range(6)}] * 2, 6, 6, [0, 1, 2], [6, 3], 10),
    ]
    for name, plans, T, V, durations, lens, max_sym in scen:
        n_dur = len(durations)
        d = V + n_dur
        enc = _plan_enc(plans, T, V, durations)
        W = np.eye(V, d, dtype=np.float32)
        W_dur = np.eye(n_dur, d, k=V, dtype=np.float32)
        P = np.zeros((V, d), np.float32)
        Q = np.zeros((7, d), np.float32)
        c = dict(enc=enc, W=W, W_dur=W_dur, P=P, Q=Q, in_lens=np.asarray(lens, np.int32))
        hyps, durs = tdt_dec(torch.from_numpy(enc), torch.tensor(lens), _predictor(P, Q), _joint(W), _joint(W_dur),
                             max(durations), blank_id=0, max_symbols_per_frame=max_sym)
        _store(out, name, "tdt", c, 0, 1, max_sym, max(durations), hyps, durs, 1.0)
        print(f"{name}: {hyps} {durs}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="checkout of the reference repository (read-only)")
    args = ap.parse_args()
    ref = Path(args.reference)
    rnnt_dec, tdt_dec = _load(ref, "rnnt"), _load(ref, "tdt")
    out: dict[str, np.ndarray] = {}
    make_reference_scenarios(out, tdt_dec)
    make_random(out, rnnt_dec, tdt_dec)
    np.savez_compressed(HERE / "decode_golden.npz", **out)
    print("decode", len(out), "arrays")


if __name__ == "__main__":
    sys.exit(main())
