"""ctypes wrapper around the C oracle (``oracle/oracle.c``).

TEST INFRASTRUCTURE ONLY: the checker for the parity tests, ``smoke()`` and the
CPU-baseline leg of ``bench.py``. Inputs are numpy arrays (float32 activations,
int32 lengths, exactly what the CUDA path receives); outputs are float64.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_SO = _HERE / "_build" / "liboracle.so"
_lib = None

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")


def build() -> Path:
    """Compile the oracle with the committed Makefile (gcc, no other dependency)."""
    subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)
    return _SO


def _load():
    global _lib
    if _lib is None:
        if not _SO.exists():
            build()
        lib = ctypes.CDLL(str(_SO))
        vp = ctypes.c_void_p
        i = ctypes.c_int
        lib.oracle_ctc.argtypes = [_f32p, _i32p, _i32p, _i32p, vp, i, i, i, i, i, _f64p, vp, i]
        lib.oracle_ctc.restype = None
        lib.oracle_rnnt.argtypes = [_f32p, _f32p, _f32p, _i32p, _i32p, _i32p, vp, i, i, i, i, i, i, i,
                                    _f64p, _f64p, vp, vp, vp, i]
        lib.oracle_rnnt.restype = None
        lib.oracle_tdt.argtypes = [_f32p, _f32p, _f32p, _f32p, _i32p, _i32p, _i32p, _i32p, i, ctypes.c_double, vp,
                                   i, i, i, i, i, i, i, _f64p, _f64p, vp, vp, vp, vp, i]
        lib.oracle_tdt.restype = None
        _lib = lib
    return _lib


def _threads(n):
    return int(n) if n else (os.cpu_count() or 1)


def _f32(x):
    return np.ascontiguousarray(np.asarray(x, dtype=np.float32))


def _i32(x):
    return np.ascontiguousarray(np.asarray(x, dtype=np.int32))


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def ctc(log_probs, targets, in_lens, tgt_lens, grad_loss=None, zero_infinity=False, nthreads=None):
    """Returns (loss (B,), grad_logits (B,T,V) or None)."""
    lp = _f32(log_probs)
    B, T, V = lp.shape
    tg = _i32(targets).reshape(B, -1)
    S = tg.shape[1]
    loss = np.zeros(B, np.float64)
    gl = None if grad_loss is None else _f32(grad_loss)
    g = None if gl is None else np.zeros((B, T, V), np.float64)
    _load().oracle_ctc(lp, tg, _i32(in_lens), _i32(tgt_lens), _ptr(gl), B, T, V, S, int(bool(zero_infinity)), loss,
                       _ptr(g), _threads(nthreads))
    return loss, g


def rnnt(enc, dec, W, targets, in_lens, tgt_lens, blank=0, grad_loss=None, nthreads=None):
    """Returns dict(loss, log_prob[, d_enc, d_dec, dW])."""
    enc, dec, W = _f32(enc), _f32(dec), _f32(W)
    B, T, d = enc.shape
    U = dec.shape[1]
    V = W.shape[0]
    tg = _i32(targets).reshape(B, -1)
    if tg.shape[1] == 0:
        tg = np.zeros((B, 1), np.int32)
    S = tg.shape[1]
    out = {"loss": np.zeros(B), "log_prob": np.zeros(B)}
    gl = None if grad_loss is None else _f32(grad_loss)
    if gl is not None:
        out["d_enc"] = np.zeros((B, T, d))
        out["d_dec"] = np.zeros((B, U, d))
        out["dW"] = np.zeros((V, d))
    _load().oracle_rnnt(enc, dec, W, tg, _i32(in_lens), _i32(tgt_lens), _ptr(gl), B, T, U, V, d, S, int(blank),
                        out["loss"], out["log_prob"], _ptr(out.get("d_enc")), _ptr(out.get("d_dec")),
                        _ptr(out.get("dW")), _threads(nthreads))
    return out


def tdt(enc, dec, W, W_dur, targets, in_lens, tgt_lens, durations, blank=0, sigma=0.0, grad_loss=None,
        nthreads=None):
    """Returns dict(loss, log_prob[, d_enc, d_dec, dW, dW_dur])."""
    enc, dec, W, W_dur = _f32(enc), _f32(dec), _f32(W), _f32(W_dur)
    B, T, d = enc.shape
    U = dec.shape[1]
    V = W.shape[0]
    Dn = W_dur.shape[0]
    dur = _i32(durations)
    assert dur.shape[0] == Dn
    tg = _i32(targets).reshape(B, -1)
    if tg.shape[1] == 0:
        tg = np.zeros((B, 1), np.int32)
    S = tg.shape[1]
    out = {"loss": np.zeros(B), "log_prob": np.zeros(B)}
    gl = None if grad_loss is None else _f32(grad_loss)
    if gl is not None:
        out["d_enc"] = np.zeros((B, T, d))
        out["d_dec"] = np.zeros((B, U, d))
        out["dW"] = np.zeros((V, d))
        out["dW_dur"] = np.zeros((Dn, d))
    _load().oracle_tdt(enc, dec, W, W_dur, tg, _i32(in_lens), _i32(tgt_lens), dur, Dn, float(sigma), _ptr(gl), B, T,
                       U, V, d, S, int(blank), out["loss"], out["log_prob"], _ptr(out.get("d_enc")),
                       _ptr(out.get("d_dec")), _ptr(out.get("dW")), _ptr(out.get("dW_dur")), _threads(nthreads))
    return out
