"""Loads the native libraries built in-tree by ``asr_b200.build``.

There is no fallback: if the CUDA extension is missing, importing the loss
modules raises, so a run can never silently compute the loss elsewhere.
"""

from __future__ import annotations

import ctypes
import os
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


# Default device-memory budget of the logit stash (see logit_stash_budget).
DEFAULT_STASH_GIB = 32.0


def logit_stash_budget() -> int:
    """Bytes the transducer losses may spend on the logit stash of one forward
    (kept until its backward): ASR_B200_LOGIT_STASH_GB (GiB; 0 turns the stash
    off, so the backward recomputes the logits GEMM), default 32 GiB. A stash
    needs about 2 KB per lattice node at V = 1024 in the bf16 mode (4 KB in the
    fp32 mode); nodes past the budget are recomputed."""
    v = os.environ.get("ASR_B200_LOGIT_STASH_GB")
    gib = DEFAULT_STASH_GIB if v is None or v == "" else float(v)
    return max(0, int(gib * (1 << 30)))


def logit_stash_layout(B: int, T: int, U: int, V: int, n_dur: int, d: int, tf32: bool) -> tuple[int, int]:
    """(nodes, bytes per node) of the logit stash the transducer losses keep for
    a (B, T, U) batch under logit_stash_budget(): the first `nodes` compact
    lattice nodes are stashed (0 when the shape runs no tensor-core joint)."""
    lib = capi_ops()
    lib.asr_logit_stash_bytes.restype = ctypes.c_size_t
    full = int(lib.asr_logit_stash_bytes(B, T, U, V, n_dur, d, 1 if tf32 else 0))
    if full <= 512:
        return 0, 0
    per = (full - 512) // ((B * T * U + 255) // 256 * 256)
    size = min(full, logit_stash_budget())
    if size <= 512:
        return 0, per
    return (size - 512) // per // 256 * 256, per
