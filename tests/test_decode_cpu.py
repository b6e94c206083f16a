"""CPU checks of greedy decoding: the numpy oracle against the golden vectors
produced by the reference's own decoders, and the host-side argument checks of
the C-ABI and of the Python decoders (nothing here launches a kernel)."""

import ctypes

import numpy as np
import pytest
import torch

from asr_b200 import _lib
from oracle import greedy
from tests.decode_cases import DECODE, expected, params


@pytest.mark.parametrize("name", sorted(DECODE))
def test_greedy_oracle_matches_reference(name):
    c = DECODE[name]
    blank, sos, max_sym, max_duration = params(c)
    want_hyps, want_durs = expected(c)
    predict = greedy.table_predictor(c["P"], c["Q"])
    if str(c["kind"]) == "rnnt":
        hyps = greedy.greedy_rnnt(c["enc"], c["in_lens"], predict, c["W"], blank, sos, max_sym)
        assert hyps == want_hyps
    else:
        hyps, durs = greedy.greedy_tdt(c["enc"], c["in_lens"], predict, c["W"], c["W_dur"], max_duration, blank, sos,
                                       max_sym)
        assert hyps == want_hyps
        assert durs == want_durs


def test_golden_cases_cover_the_edges():
    kinds = {str(c["kind"]) for c in DECODE.values()}
    assert kinds == {"rnnt", "tdt"}
    assert any(0 in c["in_lens"].tolist() for c in DECODE.values())          # empty utterance
    assert any(params(c)[0] != 0 for c in DECODE.values())                   # blank not at 0
    assert any(params(c)[2] == 1 for c in DECODE.values())                   # one symbol per frame
    assert any(c["W"].shape[0] > 1024 for c in DECODE.values())              # more than one vocab tile
    assert any(c["W"].shape[1] % 4 for c in DECODE.values())                 # joint dim not a multiple of 4
    # every frame reaching max_symbols_per_frame and being forced forward
    assert any(len(expected(c)[0][0]) == params(c)[2] * int(c["in_lens"][0]) for c in DECODE.values())


def _scan(lib, **kw):
    f = lib.asr_greedy_scan
    f.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int] + [ctypes.c_void_p] * 3 + [ctypes.c_int] + [
        ctypes.c_void_p] * 4 + [ctypes.c_int] * 10 + [ctypes.c_void_p]
    a = dict(enc=0x1000, pred=0x1000, wt=0x1000, ldw=8, wdur=None, lens=0x1000, active=None, n_active=0,
             state=0x1000, prefix=0x1000, durs=None, report=0x1000, B=2, T=4, d=8, V=6, n_dur=0, blank=0, max_sym=10,
             hyp_cap=40, dur_cap=40, max_windows=0)
    a.update(kw)
    return f(*a.values(), None)


def test_scan_rejects_bad_arguments_on_host():
    lib = _lib.capi()
    assert _scan(lib, blank=6) == 1            # blank outside the vocabulary
    assert _scan(lib, ldw=6) == 1              # leading dimension not a multiple of 4
    assert _scan(lib, ldw=4) == 1              # leading dimension below V
    assert _scan(lib, wt=0x1004) == 1          # transposed weight not 16-byte aligned
    assert _scan(lib, n_dur=3) == 1            # TDT without duration weight / buffer
    assert _scan(lib, d=5000) == 3             # joint dim beyond the shared-memory tile
    assert _scan(lib, B=0, enc=None) == 0      # empty batch: nothing to do
    assert _scan(lib, active=0x1000, n_active=0, enc=None) == 0  # empty active list
    assert _scan(lib, active=0x1000, n_active=3) == 1            # longer than the batch
    assert _scan(lib, max_windows=-1) == 1                       # negative window budget


def test_pack_and_init_reject_bad_arguments_on_host():
    lib = _lib.capi()
    lib.asr_greedy_pack_weights.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                            ctypes.c_int, ctypes.c_void_p]
    assert lib.asr_greedy_pack_weights(0x1000, 6, 8, 0x1000, 6, None) == 1
    assert lib.asr_greedy_pack_weights(None, 6, 8, 0x1000, 8, None) == 1
    lib.asr_greedy_init.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                    ctypes.c_void_p]
    assert lib.asr_greedy_init(None, None, -1, 4, 1, None) == 1
    assert lib.asr_greedy_init(None, None, 0, 4, 1, None) == 0


def test_decoders_reject_cpu_tensors():
    """Decoding has a CUDA kernel only: CPU inputs fail loudly (no CPU fallback)."""
    from asr_b200.decode import rnnt, tdt

    enc = torch.zeros(1, 3, 4)
    W = torch.zeros(5, 4)
    pred = lambda tok: torch.zeros(tok.shape[0], tok.shape[1], 4)  # noqa: E731
    with pytest.raises(RuntimeError, match="CUDA"):
        rnnt.greedy_decode(enc, torch.tensor([3]), pred, W)
    with pytest.raises(RuntimeError, match="CUDA"):
        tdt.greedy_decode(enc, torch.tensor([3]), pred, W, torch.zeros(3, 4), 2)


def test_joint_argument_forms():
    from asr_b200.decode._greedy import joint_weight

    lin = torch.nn.Linear(4, 6, bias=False)
    assert joint_weight(lin, "joint").shape == (6, 4)
    assert joint_weight(lin.weight, "joint").shape == (6, 4)
    with pytest.raises(ValueError, match="bias"):
        joint_weight(torch.nn.Linear(4, 6), "joint")
    with pytest.raises(TypeError):
        joint_weight(lambda e, p: e, "joint")
