"""Builds the native libraries in-tree for sm_100a (B200).

  asr_b200/lib/libasr_b200.so   kernels + the C ABI of include/asr_b200.h
                                (no torch dependency; loadable from any FFI)
  asr_b200/_C.abi3.so           the same kernels + the PyTorch stable-ABI shim
                                registering the asr::* ops (drop-in `_C` for the
                                reference's Python loss modules)

Run ``python -m asr_b200.build`` (or ``__graft_entry__.build()``). nvcc
cross-compiles without a GPU. Objects are cached in ``_build/`` by source
timestamp.
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD = ROOT / "_build"
LIB_DIR = PKG / "lib"
CAPI_SO = LIB_DIR / "libasr_b200.so"
OPS_SO = PKG / "_C.abi3.so"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [*ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-Xptxas", "-warn-spills", f"-I{INCLUDE}", f"-I{CSRC}"]
CU_SOURCES = ["lattice.cu", "ctc.cu", "dp_lattice.cu", "joint_simt.cu", "joint_tc.cu", "capi.cu",
              "profiler.cu", "noalloc.cu", "decode.cu", "ctc_head.cu", "ctc_beam.cu"]
HEADERS = ["common.cuh", "dp.cuh", "joint.cuh", "profiler.cuh", "tc_common.cuh"]


def _torch_paths():
    import torch

    base = Path(torch.__file__).resolve().parent
    return base / "include", base / "lib"


def _stale(out: Path, deps: list[Path]) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str]):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {cmd[0]} ... {cmd[-1]}")
    return r.stdout + r.stderr


def build(verbose: bool = False) -> dict[str, Path]:
    BUILD.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    headers = [CSRC / h for h in HEADERS] + [INCLUDE / "asr_b200.h"]
    jobs = []
    objs = []
    for src in CU_SOURCES:
        s = CSRC / src
        o = BUILD / (s.stem + ".o")
        objs.append(o)
        if _stale(o, [s, *headers, Path(__file__)]):
            jobs.append([NVCC, *NVCC_FLAGS, "-c", str(s), "-o", str(o)])
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        for log in ex.map(_run, jobs):
            if verbose and log.strip():
                print(log)
    if _stale(CAPI_SO, objs):
        _run([NVCC, *ARCH, "-shared", "-Xlinker", "-Bsymbolic", "-o", str(CAPI_SO), *map(str, objs)])
    tinc, tlib = _torch_paths()
    ops_o = BUILD / "ops.o"
    if _stale(ops_o, [CSRC / "ops.cpp", INCLUDE / "asr_b200.h"]):
        _run(["g++", "-O2", "-fPIC", "-std=c++17", "-DTORCH_TARGET_VERSION=0x020b000000000000",
              "-DPy_LIMITED_API=0x030c0000", "-DUSE_CUDA", f"-I{tinc}", f"-I{INCLUDE}", "-c", str(CSRC / "ops.cpp"), "-o",
              str(ops_o)])
    if _stale(OPS_SO, [ops_o, *objs]):
        _run([NVCC, *ARCH, "-shared", "-Xlinker", "-Bsymbolic", "-o", str(OPS_SO), str(ops_o), *map(str, objs),
              f"-L{tlib}", "-ltorch_cuda", "-ltorch_cpu", "-lc10", "-Xlinker", f"-rpath={tlib}"])
    return {"capi": CAPI_SO, "ops": OPS_SO}


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
