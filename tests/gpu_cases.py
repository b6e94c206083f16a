"""Seeded synthetic inputs shared by the GPU parity tests, smoke() and the bench.

Shapes and value distributions follow the reference's synthetic configurations
(encoder/predictor activations ~N(0, 1/d), Xavier-uniform joint weights,
uniform lengths and labels); a numpy Generator seeds every tensor group.
"""

from __future__ import annotations

import numpy as np


def xavier(rng, rows, cols):
    bound = np.sqrt(6.0 / (rows + cols))
    return rng.uniform(-bound, bound, size=(rows, cols)).astype(np.float32)


def transducer_case(seed, B, T_rng, U_rng, V, d, n_dur=0, act_std=None, w_scale=1.0, fixed_T=None):
    """Returns a dict of numpy inputs; U_rng bounds the target length (labels)."""
    rng = np.random.default_rng(seed)
    lrng = np.random.default_rng(seed + 1)
    in_lens = (np.full(B, fixed_T) if fixed_T else lrng.integers(T_rng[0], T_rng[1] + 1, size=B)).astype(np.int32)
    tgt_lens = lrng.integers(U_rng[0], U_rng[1] + 1, size=B).astype(np.int32)
    T = int(in_lens.max())
    U = int(tgt_lens.max()) + 1
    std = act_std if act_std is not None else 1.0 / np.sqrt(d)
    case = {
        "enc": (rng.standard_normal((B, T, d)) * std).astype(np.float32),
        "dec": (rng.standard_normal((B, U, d)) * std).astype(np.float32),
        "W": xavier(rng, V, d) * w_scale,
        "targets": rng.integers(1, V, size=(B, max(U - 1, 1))).astype(np.int32),
        "in_lens": in_lens,
        "tgt_lens": tgt_lens,
        "grad_loss": np.ones(B, np.float32),
    }
    if n_dur:
        case["W_dur"] = xavier(rng, n_dur, d) * w_scale
        case["durations"] = np.arange(n_dur, dtype=np.int32)
    return case


def ctc_case(seed, B, T_rng, V, S_rng):
    rng = np.random.default_rng(seed)
    lrng = np.random.default_rng(seed + 1)
    in_lens = lrng.integers(T_rng[0], T_rng[1] + 1, size=B).astype(np.int32)
    tgt_lens = lrng.integers(S_rng[0], S_rng[1] + 1, size=B).astype(np.int32)
    T, S = int(in_lens.max()), int(tgt_lens.max())
    return {
        "logits": rng.standard_normal((B, T, V)).astype(np.float32),
        "targets": rng.integers(1, V, size=(B, S)).astype(np.int32),
        "in_lens": in_lens,
        "tgt_lens": tgt_lens,
        "grad_loss": np.ones(B, np.float32),
    }


def config_draws():
    """Seeded draws with the shapes and distributions of BASELINE configs 1-5
    (fewer utterances, so that the float64 oracle finishes in seconds): config 1
    CTC char, 2 RNN-T char (T up to 400, U up to 150), 3 TDT BPE-1024, 4 RNN-T
    BPE-1024 with d = 1024 and T = 400, 5 the long end of the sharded TDT
    workload (T 450-500, U 100-120)."""
    c1 = ctc_case(61, 8, (150, 200), 29, (20, 60))
    c1["kind"] = "ctc"
    c2 = transducer_case(62, 4, (300, 400), (120, 150), 30, 640)
    c2["kind"] = "rnnt"
    c3 = transducer_case(63, 3, (300, 400), (60, 80), 1024, 640, n_dur=5)
    c3.update(kind="tdt", sigma=0.05)
    c4 = transducer_case(64, 2, None, (40, 100), 1024, 1024, fixed_T=400)
    c4["kind"] = "rnnt"
    c5 = transducer_case(65, 4, (450, 500), (100, 120), 1024, 640, n_dur=5)
    c5.update(kind="tdt", sigma=0.05)
    return {"c1_ctc": c1, "c2_rnnt_char": c2, "c3_tdt_bpe": c3, "c4_rnnt_d1024": c4, "c5_tdt_long": c5}
