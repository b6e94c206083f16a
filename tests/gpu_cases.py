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
