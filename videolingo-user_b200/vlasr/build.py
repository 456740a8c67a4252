"""Build libvlasr.so (the sm_100a kernels + C ABI) in-tree with nvcc.

Usage:  python -m vlasr.build   (from videolingo-user_b200/)  or  build_library()

Every .cu under ../csrc is compiled for sm_100a only
(-gencode arch=compute_100a,code=sm_100a) with -lineinfo, and linked into
vlasr/libvlasr.so next to this file, so the library travels with the source
tree instead of living in a JIT cache.
"""

from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
ROOT = PKG_DIR.parent                      # videolingo-user_b200/
CSRC = ROOT / "csrc"
INCLUDE = ROOT.parent / "include"          # repo-level public headers
LIB_PATH = PKG_DIR / "libvlasr.so"
BUILD_DIR = ROOT / "_build"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-warn-spills",
]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; CUDA 12.8+ is required to build libvlasr")
    return cand


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _fingerprint() -> str:
    h = hashlib.sha256()
    for p in sorted(list(CSRC.glob("*")) + list(INCLUDE.glob("*.h"))):
        if p.is_file():
            h.update(p.name.encode())
            h.update(p.read_bytes())
    h.update(" ".join(ARCH_FLAGS + NVCC_FLAGS).encode())
    return h.hexdigest()


def build_library(force: bool = False, verbose: bool = False) -> Path:
    """Compile and link libvlasr.so; skip when sources are unchanged."""
    stamp = PKG_DIR / ".libvlasr.stamp"
    fp = _fingerprint()
    if not force and LIB_PATH.exists() and stamp.exists() and stamp.read_text() == fp:
        return LIB_PATH
    # Regenerate the mel constant tables (idempotent; rewrites only on change).
    subprocess.run([sys.executable, str(CSRC / "gen_mel_tables.py")], check=True)
    BUILD_DIR.mkdir(exist_ok=True)
    # Shared inputs of every object: the headers, generated tables and flags.
    shared = hashlib.sha256()
    for q in sorted([*CSRC.glob("*.cuh"), *CSRC.glob("*.h"), *CSRC.glob("*.inc"),
                     *INCLUDE.glob("*.h")]):
        shared.update(q.name.encode())
        shared.update(q.read_bytes())
    shared.update(" ".join(ARCH_FLAGS + NVCC_FLAGS).encode())

    def compile_one(src: Path) -> str:
        """Compile one source unless its object is up to date (same source,
        headers and flags as when it was built)."""
        obj = BUILD_DIR / (src.stem + ".o")
        key = hashlib.sha256(shared.digest() + src.read_bytes()).hexdigest()
        sig = obj.with_suffix(".o.sha")
        if not force and obj.exists() and sig.exists() and sig.read_text() == key:
            return str(obj)
        cmd = [nvcc(), *ARCH_FLAGS, *NVCC_FLAGS, "-I", str(INCLUDE), "-I", str(CSRC),
               "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        sig.write_text(key)
        return str(obj)

    from concurrent.futures import ThreadPoolExecutor
    with ThreadPoolExecutor(max_workers=max(1, min(len(sources()), os.cpu_count() or 1))) as pool:
        objs = list(pool.map(compile_one, sources()))
    tmp = LIB_PATH.with_suffix(".so.tmp")
    link = [nvcc(), *ARCH_FLAGS, "-shared", "-o", str(tmp), *objs]
    if verbose:
        print(" ".join(link), flush=True)
    subprocess.run(link, check=True)
    os.replace(tmp, LIB_PATH)
    stamp.write_text(fp)
    return LIB_PATH


if __name__ == "__main__":
    print(build_library(force="--force" in sys.argv, verbose=True))
