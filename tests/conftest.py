"""Shared pytest setup.

* `-m gpu` tests need a CUDA device and the built libvlasr.so; they call the
  product through its C ABI (via the vlasr ctypes wrapper) and compare with
  the CPU oracle (oracle/) and, where built, the reference's own kernels
  (oracle/_ref/libvlref.so).
* everything else runs on a CPU-only host.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
PKG = REPO / "videolingo-user_b200"
for p in (str(REPO), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = REPO / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built libvlasr.so")


def cuda_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:  # noqa: BLE001
        return False


@pytest.fixture(scope="session")
def dev():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("gpu test selected but no CUDA device is visible")
    import vlasr
    vlasr.load()  # fail loudly if the library is missing
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def ref_kernels():
    """The reference's compiled CUDA kernels (oracle/_ref), or skip."""
    import oracle
    lib = oracle.load_reference_kernels()
    if lib is None:
        pytest.skip("oracle/_ref/libvlref.so not built (reference sources absent at build time)")
    return lib


@pytest.fixture(scope="session")
def glmasr_ckpt(tmp_path_factory):
    """A seeded synthetic checkpoint with the full official GLM-ASR-Nano
    inventory (audio tower, projector, 28-layer text model, 59264-token
    vocabulary; ~4.5 GB), written once per test session."""
    from vlasr.checkpoint import AsrModelConfig
    from vlasr.synth import write_synthetic_checkpoint
    d = tmp_path_factory.mktemp("glmasr_full")
    write_synthetic_checkpoint(d, AsrModelConfig(), seed=11)
    return d
