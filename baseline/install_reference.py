"""Installs the reference (samgd/asr) into baseline/_ref for the GPU baselines.

The reference's own build is run unmodified, as `pip install --target` runs
it, from a scratch copy of the checkout (its build writes into the source tree)
with TORCH_CUDA_ARCH_LIST=10.0a, so that its CUDA loss op (asr.loss._C,
src/asr/loss/csrc/*) is compiled for sm_100a:

    python -m pip install --no-index --no-build-isolation --no-deps \
        --find-links /opt/wheelhouse --target baseline/_ref <copy of the checkout>

In this image that command stops at the reference's second extension,
asr.decode._C, whose -fopenmp link cannot find gcc's libgomp.spec; the loss op
has been built by then. When that is the only failure, the package tree the
build produced (its Python modules and asr/loss/_C.abi3.so) is placed in
baseline/_ref/asr, which is what the install writes for the loss path. The op
is loaded only in processes that do not load asr_b200's own op library (both
register the asr:: namespace); baseline/ref_worker.py is that process.

    python baseline/install_reference.py [REFERENCE_DIR]

REFERENCE_DIR defaults to ASR_REFERENCE_DIR, else a `reference` directory
beside this repository.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
TARGET = HERE / "_ref"


def installed() -> bool:
    return any((TARGET / "asr" / "loss").glob("_C*.so"))


def install(ref: str | None = None, quiet: bool = True) -> bool:
    ref = ref or os.environ.get("ASR_REFERENCE_DIR") or str(ROOT.parent / "reference")
    if not (Path(ref) / "src" / "asr" / "loss" / "csrc" / "tdt.cu").exists():
        return False
    with tempfile.TemporaryDirectory(prefix="asr_ref_build_") as tmp:
        src = Path(tmp) / "src_copy"
        shutil.copytree(ref, src, ignore=shutil.ignore_patterns(".git", "build", "*.egg-info"))
        for p in src.rglob("*"):
            p.chmod(p.stat().st_mode | 0o200)
        env = dict(os.environ, TORCH_CUDA_ARCH_LIST="10.0a", MAX_JOBS=str(min(8, os.cpu_count() or 1)))
        cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--no-deps",
               "--find-links", "/opt/wheelhouse", "--target", str(TARGET), str(src)]
        r = subprocess.run(cmd, env=env, capture_output=True, text=True)
        if r.returncode == 0:
            return installed()
        built = sorted(src.glob("build/lib*/asr"))
        openmp_only = "libgomp.spec" in r.stdout + r.stderr
        if not (built and any((built[0] / "loss").glob("_C*.so")) and openmp_only):
            if not quiet:
                sys.stderr.write(r.stdout[-3000:] + r.stderr[-3000:])
            return False
        shutil.rmtree(TARGET / "asr", ignore_errors=True)
        TARGET.mkdir(parents=True, exist_ok=True)
        shutil.copytree(built[0], TARGET / "asr", ignore=shutil.ignore_patterns("csrc"))
    return installed()


if __name__ == "__main__":
    ok = install(sys.argv[1] if len(sys.argv) > 1 else None, quiet=False)
    print("reference installed in", TARGET if ok else "nothing (reference checkout or its loss op build missing)")
    sys.exit(0 if ok else 1)
