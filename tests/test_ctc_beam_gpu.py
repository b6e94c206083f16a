"""Parity of the GPU CTC decoders (asr_b200.decode.ctc) with the reference's.

Outputs are token sequences, so the bar is exact equality: with the golden
vectors made by the reference's own beam-search op, with that op itself
(oracle/_ref, when built) on fresh BPE-size draws, and with the greedy
restatement. Random float32 log-probs make exact score ties, which the
reference resolves in an unspecified order, vanishingly unlikely."""

import numpy as np
import pytest
import torch

from asr_b200.decode import ctc
from oracle import ctc_beam
from tests.decode_cases import split
from tests.golden_io import load_cases

pytestmark = pytest.mark.gpu

CASES = load_cases("ctc_beam")


@pytest.mark.parametrize("name", sorted(CASES))
def test_beam_matches_reference_golden(name):
    c = CASES[name]
    got = ctc.beam_decode(torch.tensor(c["log_probs"], device="cuda"), torch.tensor(c["in_lens"]), int(c["beam"]))
    assert got == split(c["hyp_flat"], c["hyp_lens"])


def draw(seed, B, T, V, scale=4.0, blank=1.5):
    rng = np.random.default_rng(seed)
    logits = rng.standard_normal((B, T, V)) * scale
    logits[..., 0] += scale * blank
    lp = torch.log_softmax(torch.tensor(logits, dtype=torch.float32), -1).numpy()
    return lp, rng.integers(T // 2, T + 1, size=B).astype(np.int32)


@pytest.mark.skipif(not ctc_beam.reference_available(), reason="reference op not built into oracle/_ref")
@pytest.mark.parametrize("V,W", [(1024, 32), (1024, 8), (29, 32), (300, 64)])
def test_beam_matches_reference_op(V, W):
    lp, il = draw(V + W, 4, 120, V)
    want = ctc_beam.reference_beam_decode(lp, il, W)
    assert ctc.beam_decode(torch.tensor(lp, device="cuda"), torch.tensor(il), W) == want


def test_beam_on_cpu_input_and_edge_lengths():
    lp, _ = draw(3, 3, 40, 29)
    il = np.array([0, 1, 40], np.int32)
    got = ctc.beam_decode(torch.tensor(lp), torch.tensor(il), 8)  # CPU tensor: moved to the GPU
    assert got == ctc_beam.beam_decode(lp, il, 8)
    assert got[0] == []


def test_greedy_matches_restatement():
    lp, il = draw(4, 6, 80, 64)
    assert ctc.greedy_decode(torch.tensor(lp, device="cuda"), torch.tensor(il)) == ctc_beam.greedy_decode(lp, il)
