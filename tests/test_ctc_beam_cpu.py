"""CPU checks of CTC decoding: the restatement of the reference beam search
against the golden vectors of the reference op itself, the reference op (when
built into oracle/_ref) against the restatement, and host-side C-ABI checks."""

import ctypes

import numpy as np
import pytest

from asr_b200 import _lib
from oracle import ctc_beam
from tests.decode_cases import split
from tests.golden_io import load_cases

CASES = load_cases("ctc_beam")


def expected(c):
    return split(c["hyp_flat"], c["hyp_lens"])


@pytest.mark.parametrize("name", sorted(CASES))
def test_beam_restatement_matches_reference_golden(name):
    c = CASES[name]
    if c["log_probs"].shape[2] > 64 and c["log_probs"].shape[1] * int(c["beam"]) > 2000:
        pytest.skip("pure-Python restatement is too slow for this case (the GPU test covers it)")
    assert ctc_beam.beam_decode(c["log_probs"], c["in_lens"], int(c["beam"])) == expected(c)


@pytest.mark.skipif(not ctc_beam.reference_available(), reason="reference op not built (make -C oracle ref)")
def test_reference_op_matches_restatement_on_fresh_draws():
    rng = np.random.default_rng(11)
    import torch

    lp = torch.log_softmax(torch.tensor(rng.standard_normal((3, 30, 17)) * 3, dtype=torch.float32), -1).numpy()
    il = np.array([30, 22, 9])
    for W in (1, 3, 8, 20):
        assert ctc_beam.reference_beam_decode(lp, il, W) == ctc_beam.beam_decode(lp, il, W)


def test_greedy_restatement():
    lp = np.log(np.array([[[0.1, 0.8, 0.1], [0.1, 0.8, 0.1], [0.8, 0.1, 0.1], [0.1, 0.1, 0.8], [0.1, 0.8, 0.1]]],
                         np.float32))
    assert ctc_beam.greedy_decode(lp, [5]) == [[1, 2, 1]]
    assert ctc_beam.greedy_decode(lp, [3]) == [[1]]


def test_c_abi_rejects_bad_arguments_on_host():
    lib = _lib.capi()
    f = lib.asr_ctc_beam_workspace_bytes
    f.restype = ctypes.c_size_t
    assert f(2, 10, 8) > 0
    assert f(2, 10, 0) == 0 and f(2, 10, 65) == 0
    g = lib.asr_ctc_beam_decode
    P, I = ctypes.c_void_p, ctypes.c_int
    g.argtypes = [P, P, I, I, I, I, P, P, P, ctypes.c_size_t, P]
    fake = 0x1000
    assert g(fake, fake, 2, 10, 29, 65, fake, fake, fake, 1 << 20, None) == 3   # beam too wide
    assert g(fake, fake, 2, 10, 9000, 8, fake, fake, fake, 1 << 20, None) == 3  # vocabulary too large
    assert g(fake, fake, 2, 10, 29, 8, fake, fake, fake, 16, None) == 2         # workspace too small
    assert g(None, fake, 2, 10, 29, 8, fake, fake, fake, 1 << 20, None) == 1
    assert g(None, None, 0, 10, 29, 8, None, None, None, 0, None) == 0          # empty batch
