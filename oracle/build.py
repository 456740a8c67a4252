"""Build the CPU oracle (liboracle.so) and, where the reference tree is
mounted, the reference-kernel harness (oracle/_ref/libvlref.so).

TEST INFRASTRUCTURE ONLY.  liboracle.so is the C restatement of the
reference algorithms (vl_oracle.c).  libvlref.so compiles the reference's own
CUDA sources in place (VideoLingo-user native/asr/src/*.cu, read where they
lie, never copied) together with ref_harness/*.cu, which re-export the
reference's anonymous-namespace kernels through extern "C" launchers so GPU
tests can run the reference implementation on the same inputs.  Both
outputs are git-ignored build products.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"
REF_DIR = HERE / "_ref"
REF_LIB = REF_DIR / "libvlref.so"
# The reference checkout: $VL_REFERENCE_SRC, else a `reference` directory
# beside this repository (its native/asr/src).  Absent on hosts that only run
# the prebuilt libraries.
REF_SRC = Path(os.environ.get("VL_REFERENCE_SRC")
               or HERE.parent.parent / "reference" / "native" / "asr" / "src")


def build_oracle(force: bool = False) -> Path:
    src = HERE / "vl_oracle.c"
    if not force and LIB.exists() and LIB.stat().st_mtime >= src.stat().st_mtime:
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    subprocess.run(["gcc", "-O2", "-fPIC", "-shared", "-mfma", "-ffp-contract=off",
                    "-o", str(tmp), str(src), "-lm"], check=True)
    os.replace(tmp, LIB)
    return LIB


def build_reference_harness(force: bool = False) -> Path | None:
    """Compile the reference kernels for sm_100a (only where its sources exist)."""
    if not REF_SRC.is_dir():
        return REF_LIB if REF_LIB.exists() else None
    harness = sorted((HERE / "ref_harness").glob("*.cu"))
    inputs = harness + sorted(REF_SRC.glob("*.cu")) + sorted(REF_SRC.glob("*.h"))
    newest = max(p.stat().st_mtime for p in inputs)
    if not force and REF_LIB.exists() and REF_LIB.stat().st_mtime >= newest:
        return REF_LIB
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    REF_DIR.mkdir(exist_ok=True)
    objs = []
    flags = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17",
             "-Xcompiler", "-fPIC", "-I", str(REF_SRC), "-w"]
    for h in harness:
        obj = REF_DIR / (h.stem + ".o")
        subprocess.run([nvcc, *flags, "-c", str(h), "-o", str(obj)], check=True)
        objs.append(str(obj))
    # model_loader.cu provides symbols engine.cu's host code references.
    obj = REF_DIR / "model_loader.o"
    subprocess.run([nvcc, *flags, "-c", str(REF_SRC / "model_loader.cu"), "-o", str(obj)],
                   check=True)
    objs.append(str(obj))
    tmp = REF_LIB.with_suffix(".so.tmp")
    subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", str(tmp),
                    *objs, "-lcublas", "-lcublasLt"], check=True)
    os.replace(tmp, REF_LIB)
    return REF_LIB


if __name__ == "__main__":
    print(build_oracle(force="--force" in sys.argv))
    print(build_reference_harness(force="--force" in sys.argv))
