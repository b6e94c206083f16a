"""Shared helpers of the greedy-decoding tests: golden case access and seeded inputs."""

import numpy as np

from tests.golden_io import load_cases

DECODE = load_cases("decode")


def split(flat, lens):
    out, i = [], 0
    for n in np.asarray(lens).tolist():
        out.append(np.asarray(flat[i: i + n]).tolist())
        i += n
    return out


def expected(c):
    hyps = split(c["hyp_flat"], c["hyp_lens"])
    durs = split(c["dur_flat"], c["dur_lens"]) if "dur_flat" in c else None
    return hyps, durs


def params(c):
    blank, sos, max_sym, max_duration = (int(x) for x in c["params"])
    return blank, sos, max_sym, max_duration


def random_decode_case(seed, B, T, V, d, n_dur, blank_bias, lo=None):
    """Inputs in the style of the golden generator: W[blank] weights a constant
    encoder direction by blank_bias, so blank wins most steps as in a trained model."""
    rng = np.random.default_rng(seed)
    enc = (rng.standard_normal((B, T, d)) * 0.8).astype(np.float32)
    enc[..., 0] = 2.0
    W = (rng.standard_normal((V, d)) / np.sqrt(d) * 3.0).astype(np.float32)
    W[0, 0] += blank_bias
    c = dict(enc=enc, W=W, P=(rng.standard_normal((V, d)) * 0.5).astype(np.float32),
             Q=(rng.standard_normal((7, d)) * 0.3).astype(np.float32),
             in_lens=rng.integers(lo if lo is not None else T // 2, T + 1, size=B).astype(np.int32))
    if n_dur:
        Wd = (rng.standard_normal((n_dur, d)) / np.sqrt(d) * 3.0).astype(np.float32)
        Wd[1, 0] += 0.5
        c["W_dur"] = Wd
    return c
