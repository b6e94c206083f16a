"""Loads the native libraries built in-tree by ``asr_b200.build``.

There is no fallback: if the CUDA extension is missing, importing the loss
modules raises, so a run can never silently compute the loss elsewhere.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import torch

_PKG = Path(__file__).resolve().parent
OPS_SO = _PKG / "_C.abi3.so"
CAPI_SO = _PKG / "lib" / "libasr_b200.so"

_ops_loaded = False
_capi = None


def load_ops() -> None:
    """Registers the ``torch.ops.asr.*`` operators (idempotent)."""
    global _ops_loaded
    if _ops_loaded:
        return
    if not OPS_SO.exists():
        raise RuntimeError(f"asr_b200 CUDA extension not built: {OPS_SO} is missing (run `python -m asr_b200.build`)")
    torch.ops.load_library(str(OPS_SO))
    _ops_loaded = True


def capi_ops() -> ctypes.CDLL:
    """ctypes view of the op library itself (the kernels torch.ops.asr.* run), for
    the diagnostics entry points (asr_profiler_*, asr_joint_path)."""
    load_ops()
    return ctypes.CDLL(str(OPS_SO))


def joint_uses_tensor_cores(V: int, n_dur: int, d: int, tf32: bool = True) -> bool:
    """True when the tcgen05 joint runs for this shape: bf16 operands with
    tf32=True, split fp32 operands (three bf16 products) with tf32=False."""
    return bool(capi_ops().asr_joint_path(1 if tf32 else 0, V, n_dur, d))


def capi() -> ctypes.CDLL:
    """The C-ABI library (include/asr_b200.h) for FFI callers and tests."""
    global _capi
    if _capi is None:
        if not CAPI_SO.exists():
            raise RuntimeError(f"asr_b200 C-ABI library not built: {CAPI_SO} is missing")
        _capi = ctypes.CDLL(str(CAPI_SO))
    return _capi
