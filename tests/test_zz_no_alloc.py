"""asr_tdt_forward_noalloc: the TDT forward for callers that cannot allocate
device memory (a bare FFI host with no device allocator, a service that reserves
all GPU memory at start-up, code where a cudaMalloc would synchronise the device).
It takes no workspace and uses a fixed scratch array compiled into the library.

Called through the C ABI (ctypes on libasr_b200.so) and checked against the
regular asr_tdt_forward, which gets a caller-provided workspace, on two calls
in a row (the scratch keeps the previous call's contents), with the loss
tolerance of the other parity tests. The file sorts last so a run that stops at
the first failure has already run every other test; it also passes alone.
"""

import ctypes

import numpy as np
import pytest
import torch

from asr_b200 import _lib
from tests.golden_io import load_cases

pytestmark = pytest.mark.gpu

LOSS_RTOL = 1e-5
LOSS_ATOL = 1e-5
TDT = load_cases("tdt")


def P(t):
    return ctypes.c_void_p(t.data_ptr())


def _outputs(B, T, U, Dn):
    f32 = dict(device="cuda", dtype=torch.float32)
    return {
        "loss": torch.full((B,), float("nan"), **f32),
        "alpha": torch.full((B, T + 1, U), float("nan"), device="cuda", dtype=torch.float64),
        "lpb": torch.full((2, B, T, U), float("nan"), **f32),
        "lpy": torch.full((B, T, U), float("nan"), **f32),
        "lpd": torch.full((B, T, U, Dn), float("nan"), **f32),
        "log_prob": torch.full((B,), float("nan"), **f32),
    }


def _run(lib, c, tf32, noalloc):
    B, T, d = c["enc"].shape
    U = c["dec"].shape[1]
    V = c["W"].shape[0]
    Dn = c["W_dur"].shape[0]
    S = c["targets"].shape[1]
    t = {k: torch.as_tensor(np.ascontiguousarray(c[k]), device="cuda")
         for k in ("enc", "dec", "W", "W_dur", "targets", "in_lens", "tgt_lens", "durations")}
    o = _outputs(B, T, U, Dn)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    md = int(c["durations"].max())
    hz = int((c["durations"] == 0).any())
    head = [P(t["enc"]), P(t["dec"]), P(t["W"]), P(t["W_dur"]), P(t["targets"]), P(t["in_lens"]), P(t["tgt_lens"]),
            P(t["durations"]), Dn, md, hz, B, T, U, V, d, S, 0, ctypes.c_float(float(c["sigma"])), tf32,
            P(o["loss"]), P(o["alpha"]), P(o["lpb"]), P(o["lpy"]), P(o["lpd"]), P(o["log_prob"])]
    if noalloc:
        rc = lib.asr_tdt_forward_noalloc(*head, stream)
    else:
        lib.asr_tdt_workspace_bytes.restype = ctypes.c_size_t
        wsb = lib.asr_tdt_workspace_bytes(B, T, U, V, Dn, d, tf32, 0)
        ws = torch.empty(wsb, dtype=torch.uint8, device="cuda")
        rc = lib.asr_tdt_forward(*head, P(ws), ctypes.c_size_t(wsb), stream)
    assert rc == 0, f"rc={rc}"
    torch.cuda.synchronize()
    n = int((c["in_lens"].astype(np.int64) * (c["tgt_lens"] + 1)).sum())
    na = int(((c["in_lens"].astype(np.int64) + 1) * (c["tgt_lens"] + 1)).sum())
    cap = B * T * U
    return {
        "loss": o["loss"].cpu().numpy(), "log_prob": o["log_prob"].cpu().numpy(),
        "alpha": o["alpha"].view(-1)[:na].cpu().numpy(),
        "lpb": o["lpb"].view(-1)[:n].cpu().numpy(), "lse": o["lpb"].view(-1)[cap:cap + n].cpu().numpy(),
        "lpy": o["lpy"].view(-1)[:n].cpu().numpy(), "lpd": o["lpd"].view(-1)[:n * Dn].cpu().numpy(),
    }


@pytest.mark.parametrize("tf32", [0, 1])
@pytest.mark.parametrize("name", ["variable_lens_s02", "wider", "empty_target_in_batch"])
def test_noalloc_forward_matches_workspace_forward_twice(name, tf32):
    lib = _lib.capi()
    c = TDT[name]
    want = _run(lib, c, tf32, noalloc=False)
    for _ in range(2):
        got = _run(lib, c, tf32, noalloc=True)
        np.testing.assert_allclose(got["loss"], want["loss"], rtol=LOSS_RTOL, atol=LOSS_ATOL)
        np.testing.assert_allclose(got["log_prob"], want["log_prob"], rtol=LOSS_RTOL, atol=LOSS_ATOL)
        for k in ("alpha", "lpb", "lse", "lpy", "lpd"):
            np.testing.assert_allclose(got[k], want[k], rtol=LOSS_RTOL, atol=LOSS_ATOL, err_msg=k)


def test_noalloc_rejects_problems_beyond_its_scratch():
    lib = _lib.capi()
    null = ctypes.c_void_p(0)
    limit = 4 << 20
    lib.asr_tdt_workspace_bytes.restype = ctypes.c_size_t
    # with tf32 = 0 the forward's scratch is the per-utterance lattice bookkeeping
    # (~16 bytes per utterance), so a batch of 400k short utterances needs more than
    # the array holds (with tf32 = 1 the bf16 weights and hidden rows come on top)
    B, T, U, V, Dn, d = 400_000, 2, 2, 16, 5, 8
    assert lib.asr_tdt_workspace_bytes(B, T, U, V, Dn, d, 0, 0) > limit
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.asr_tdt_forward_noalloc(*([null] * 8), Dn, 4, 1, B, T, U, V, d, U - 1, 0, ctypes.c_float(0.0), 0,
                                     *([null] * 6), stream)
    assert rc == 5
    lib.asr_status_string.restype = ctypes.c_char_p
    assert b"scratch" in lib.asr_status_string(rc)


def test_noalloc_forward_takes_no_device_memory():
    """After a first call in this context (which loads the module and so may map
    memory), further calls leave the device's free memory as it was: no
    cudaMalloc, no pool growth. Both joint paths. torch's caching allocator holds
    the inputs and outputs, which are warmed up before the measurement."""
    lib = _lib.capi()
    c = TDT["wider"]
    for tf32 in (0, 1):
        _run(lib, c, tf32, noalloc=True)
        torch.cuda.synchronize()
        free0, _ = torch.cuda.mem_get_info()
        for _ in range(3):
            _run(lib, c, tf32, noalloc=True)
        torch.cuda.synchronize()
        free1, _ = torch.cuda.mem_get_info()
        assert free1 >= free0, f"tf32={tf32}: free device memory fell by {free0 - free1} bytes"
