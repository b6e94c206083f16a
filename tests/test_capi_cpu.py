"""CPU checks of the native boundary: the C-ABI library loads and exports every
declared entry point, host-side argument checks reject bad calls without
touching a GPU, and the op shim registers the reference's exact schemas."""

import ctypes
import re
from pathlib import Path

import pytest
import torch

from asr_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "asr_b200.h"

# Schemas of the reference ops (src/asr/loss/csrc/*_bindings.cpp).
REFERENCE_SCHEMAS = {
    "ctc_alpha": "asr::ctc_alpha(Tensor log_probs, Tensor targets, Tensor in_lens, Tensor tgt_lens) -> (Tensor, Tensor)",
    "ctc_grad": "asr::ctc_grad(Tensor alpha, Tensor log_Z, Tensor log_probs, Tensor targets, Tensor in_lens, "
    "Tensor tgt_lens, Tensor grad_loss, bool zero_infinity) -> Tensor",
    "rnnt_forward": "asr::rnnt_forward(Tensor encoder, Tensor decoder, Tensor joint_W, Tensor targets, Tensor in_lens, "
    "Tensor tgt_lens, int blank_idx, int tf32) -> (Tensor, Tensor, Tensor, Tensor, Tensor)",
    "rnnt_backward": "asr::rnnt_backward(Tensor encoder, Tensor decoder, Tensor joint_W, Tensor targets, "
    "Tensor in_lens, Tensor tgt_lens, int blank_idx, Tensor alpha, Tensor log_P_blank, Tensor log_P_y, "
    "Tensor log_prob, Tensor grad_loss, int tf32) -> (Tensor, Tensor, Tensor)",
    "tdt_forward": "asr::tdt_forward(Tensor encoder, Tensor decoder, Tensor joint_W, Tensor joint_W_dur, "
    "Tensor targets, Tensor in_lens, Tensor tgt_lens, Tensor durations, int max_duration, int has_zero, "
    "int blank_idx, float sigma, int tf32) -> (Tensor, Tensor, Tensor, Tensor, Tensor, Tensor)",
    "tdt_backward": "asr::tdt_backward(Tensor encoder, Tensor decoder, Tensor joint_W, Tensor joint_W_dur, "
    "Tensor targets, Tensor in_lens, Tensor tgt_lens, Tensor durations, int max_duration, int has_zero, "
    "int blank_idx, Tensor alpha, Tensor log_P_blank, Tensor log_P_y, Tensor log_P_dur, Tensor log_prob, "
    "Tensor grad_loss, int tf32) -> (Tensor, Tensor, Tensor, Tensor)",
}


def declared_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:const char\*|int|size_t)\s+(asr_\w+)\s*\(", text, re.M)))


def test_header_declares_entry_points():
    names = declared_functions()
    for must in ("asr_ctc_alpha", "asr_ctc_grad", "asr_rnnt_forward", "asr_rnnt_backward", "asr_tdt_forward",
                 "asr_tdt_backward", "asr_rnnt_workspace_bytes", "asr_tdt_workspace_bytes"):
        assert must in names


def test_capi_exports_every_declared_symbol():
    lib = _lib.capi()
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} declared in include/asr_b200.h but not exported"


def test_status_strings_and_version():
    lib = _lib.capi()
    lib.asr_status_string.restype = ctypes.c_char_p
    assert lib.asr_status_string(0) == b"ok"
    assert b"workspace" in lib.asr_status_string(2)
    assert lib.asr_abi_version() == 2


def _ws(lib, fn, *args):
    f = getattr(lib, fn)
    f.restype = ctypes.c_size_t
    return f(*map(ctypes.c_int, args))


def test_workspace_sizes_monotone():
    lib = _lib.capi()
    small = _ws(lib, "asr_tdt_workspace_bytes", 4, 50, 10, 64, 5, 32, 0, 1)
    big = _ws(lib, "asr_tdt_workspace_bytes", 8, 50, 10, 64, 5, 32, 0, 1)
    assert 0 < small < big
    assert _ws(lib, "asr_tdt_workspace_bytes", 4, 50, 10, 64, 5, 32, 0, 0) < small
    assert _ws(lib, "asr_rnnt_workspace_bytes", 4, 0, 10, 64, 32, 0, 0) == 0  # T < 1 is invalid


def test_bf16_activation_workspace_and_dtype_checks():
    """The *_ex entry points: bf16 activations add fp32 staging to the workspace
    (gradient sums in the backward), float32 matches the plain entry points, and an
    unknown activation dtype is rejected on the host."""
    lib = _lib.capi()
    for fn, base, args in (("asr_tdt_workspace_bytes_ex", "asr_tdt_workspace_bytes", (4, 50, 10, 64, 5, 32, 0)),
                           ("asr_rnnt_workspace_bytes_ex", "asr_rnnt_workspace_bytes", (4, 50, 10, 64, 32, 0))):
        for bwd in (0, 1):
            f32 = _ws(lib, fn, *args, bwd, 0)
            assert f32 == _ws(lib, base, *args, bwd)
            assert _ws(lib, fn, *args, bwd, 1) > f32
            assert _ws(lib, fn, *args, bwd, 7) == 0
    null = ctypes.c_void_p(0)
    fake = ctypes.c_void_p(0x1000)
    args = [fake, fake, ctypes.c_int(7)] + [fake] * 4 + [ctypes.c_int(v) for v in (2, 4, 3, 5, 8, 2, 0, 0)] + \
        [fake] * 5 + [null, ctypes.c_size_t(0), null]
    assert lib.asr_rnnt_forward_ex(*args) == 1


def test_invalid_arguments_rejected_on_host():
    lib = _lib.capi()
    null = ctypes.c_void_p(0)
    # B < 0
    rc = lib.asr_ctc_alpha(null, null, null, null, -1, 4, 3, 1, null, null, null)
    assert rc == 1
    # null pointers with B > 0
    rc = lib.asr_ctc_alpha(null, null, null, null, 2, 4, 3, 1, null, null, null)
    assert rc == 1
    # blank index out of range
    args = [null] * 6 + [ctypes.c_int(v) for v in (2, 4, 3, 5, 8, 2, 7, 0)] + [null] * 5 + [null, ctypes.c_size_t(0),
                                                                                            null]
    assert lib.asr_rnnt_forward(*args) == 1
    # zero-size workspace with valid-looking pointers is a workspace error, not a launch
    fake = ctypes.c_void_p(0x1000)
    args = [fake] * 6 + [ctypes.c_int(v) for v in (2, 4, 3, 5, 8, 2, 0, 0)] + [fake] * 5 + [null, ctypes.c_size_t(0),
                                                                                            null]
    assert lib.asr_rnnt_forward(*args) == 2


def test_op_shim_registers_reference_schemas():
    _lib.load_ops()
    for name, schema in REFERENCE_SCHEMAS.items():
        got = str(getattr(torch.ops.asr, name).default._schema)
        assert got == schema, f"{name}: {got}"


def test_tdt_loss_validates_durations_on_host():
    from asr_b200.loss.tdt import tdt_loss

    enc = torch.zeros(1, 2, 4)
    dec = torch.zeros(1, 2, 4)
    W = torch.zeros(3, 4)
    tgt = torch.zeros(1, 1, dtype=torch.int32)
    ln = torch.ones(1, dtype=torch.int32)
    with pytest.raises(ValueError, match="contain 1"):
        tdt_loss(enc, dec, W, torch.zeros(2, 4), tgt, ln, ln, [0, 2])
    with pytest.raises(ValueError, match="non-negative"):
        tdt_loss(enc, dec, W, torch.zeros(2, 4), tgt, ln, ln, [-1, 1])
    with pytest.raises(ValueError, match="must equal"):
        tdt_loss(enc, dec, W, torch.zeros(3, 4), tgt, ln, ln, [0, 1])
    with pytest.raises(ValueError, match="sigma"):
        tdt_loss(enc, dec, W, torch.zeros(2, 4), tgt, ln, ln, [0, 1], sigma=-0.1)


def test_cpu_tensors_are_rejected_not_computed():
    """The ops have a CUDA kernel only: CPU inputs must fail loudly (no CPU fallback)."""
    from asr_b200.loss.rnnt import rnnt_loss

    enc = torch.zeros(1, 2, 4)
    dec = torch.zeros(1, 2, 4)
    W = torch.zeros(3, 4)
    tgt = torch.ones(1, 1, dtype=torch.int32)
    ln = torch.ones(1, dtype=torch.int32)
    with pytest.raises((RuntimeError, NotImplementedError)):
        rnnt_loss(enc, dec, W, tgt, ln, ln)
