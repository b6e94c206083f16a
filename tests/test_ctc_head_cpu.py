"""CPU checks of the fused CTC head: the float64 oracle against the golden vectors
of the reference head + loss, and host-side argument checks of the C-ABI."""

import ctypes

import numpy as np
import pytest
import torch

from asr_b200 import _lib
from oracle import ctc_head
from tests.golden_io import load_cases

CASES = load_cases("ctc_head")


def run_oracle(c):
    return ctc_head.ctc_head(c["enc"], c["g"], c["W"], c.get("b"), c["targets"], c["in_lens"], c["tgt_lens"],
                             zero_infinity=bool(c["zero_infinity"]), grad_loss=c["grad_loss"])


@pytest.mark.parametrize("name", sorted(CASES))
def test_ctc_head_oracle_matches_reference(name):
    c = CASES[name]
    out = run_oracle(c)
    # float32 RMSNorm and log-probs on both sides; the CTC recursion of the C oracle
    # reads float32 log-probs
    np.testing.assert_allclose(out["loss"], c["loss"], rtol=2e-6, atol=2e-5)
    for k in ("d_enc", "dg", "dW", "db"):
        if k in c:
            np.testing.assert_allclose(out[k], c[k], rtol=1e-4, atol=2e-6, err_msg=k)


def test_golden_cases_cover_the_edges():
    assert any("b" not in c for c in CASES.values())
    assert any(c["tgt_lens"].min() == 0 for c in CASES.values())
    assert any(int(c["zero_infinity"]) and (c["loss"] == 0).any() for c in CASES.values())
    assert any(c["W"].shape[1] % 8 for c in CASES.values())


def test_c_abi_rejects_bad_arguments_on_host():
    lib = _lib.capi()
    f = lib.asr_ctc_head_workspace_bytes
    f.restype = ctypes.c_size_t
    assert f(4, 50, 10, 64, 32, 0) > 0
    assert f(4, 50, 10, 64, 32, 7) == 0      # unknown activation dtype
    assert f(4, 0, 10, 64, 32, 0) == 0       # T < 1
    fwd = lib.asr_ctc_head_forward
    P, I = ctypes.c_void_p, ctypes.c_int
    fwd.argtypes = [P, I, P, ctypes.c_float, P, P, P, P, P] + [I] * 6 + [P, P, ctypes.c_size_t, P]
    fake = 0x1000
    # S = 600: 2S + 1 > 1024 is beyond the CTC recursion
    assert fwd(fake, 0, fake, 1e-6, fake, None, fake, fake, fake, 2, 8, 600, 16, 32, 0, fake, fake, 1 << 30,
               None) == 3
    # null loss pointer
    assert fwd(fake, 0, fake, 1e-6, fake, None, fake, fake, fake, 2, 8, 3, 16, 32, 0, None, fake, 1 << 30,
               None) == 1


def test_module_state_dict_matches_the_reference_head():
    from asr_b200.loss.ctc_head import FusedCTCHead

    head = FusedCTCHead(16, 7)
    ref = torch.nn.Sequential(torch.nn.RMSNorm(16), torch.nn.Linear(16, 7))
    assert set(head.state_dict()) == set(ref.state_dict())
    head.load_state_dict(ref.state_dict())
    x = torch.randn(2, 3, 16)
    torch.testing.assert_close(head(x), ref(x))


def test_fused_call_rejects_cpu_tensors():
    from asr_b200.loss.ctc_head import FusedCTCHead

    head = FusedCTCHead(16, 7)
    with pytest.raises(RuntimeError, match="CUDA"):
        head(torch.randn(1, 4, 16), torch.ones(1, 2, dtype=torch.int32), torch.tensor([4]), torch.tensor([2]))
