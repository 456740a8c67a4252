"""vl_logmel_noalloc: the log-mel entry point that allocates nothing.

Some callers cannot allocate device memory for this library - their GPU
memory is reserved up front by a fixed budget or arena, or they run inside
another framework's callback where allocating is not allowed - so they
cannot provide vl_logmel's workspace.  vl_logmel_noalloc keeps that scratch
in a fixed array inside the library instead.  These tests call it through
the C ABI and check it bit for bit against vl_logmel (the workspace entry
point), and against the WhisperFeatureExtractor golden features.  They pass
alone in a fresh process and after the rest of the suite.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

import vlasr
from conftest import GOLDEN
from vlasr import _lib
from vlasr.synth import audio_chunks, tone_pcm

MAX_CHUNKS = 1024  # VL_LOGMEL_NOALLOC_MAX_CHUNKS in include/vl_api.h


def test_noalloc_rejects_sizes_beyond_its_scratch():
    """Validated on the host before any CUDA call (no GPU needed)."""
    lib = vlasr.load()
    fake = 0x10000
    rc = lib.vl_logmel_noalloc(fake, MAX_CHUNKS + 1, fake * 1000000, None)
    assert rc == _lib.VL_ERR_INVALID
    msg = lib.vl_last_error().decode()
    assert str(MAX_CHUNKS) in msg and "vl_logmel" in msg
    assert lib.vl_logmel_noalloc(fake, 0, fake * 1000000, None) == _lib.VL_ERR_INVALID
    assert lib.vl_logmel_noalloc(None, 1, fake, None) == _lib.VL_ERR_INVALID


def _noalloc(lib, pcm, out, stream) -> None:
    rc = lib.vl_logmel_noalloc(ctypes.c_void_p(pcm.data_ptr()), pcm.shape[0],
                               ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(stream))
    assert rc == _lib.VL_OK, lib.vl_last_error().decode()


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_point_twice_in_a_row(dev):
    import torch

    lib = vlasr.load()
    stream = torch.cuda.current_stream(dev).cuda_stream
    # Two different inputs back to back: the second call must not be
    # affected by what the first left in the shared scratch array (the
    # chunk maxima differ), and 35 chunks cross the kernel's 32-chunk batch.
    # Both entry points run the same kernels, so the features must be
    # bit-identical.
    first = audio_chunks(35, seed=101)
    second = audio_chunks(3, seed=202) * np.float32(0.05)
    for pcm_np in (first, second):
        pcm = torch.from_numpy(pcm_np).to(dev)
        expected = vlasr.logmel(pcm)
        out = torch.full_like(expected, float("nan"))
        _noalloc(lib, pcm, out, stream)
        torch.cuda.synchronize()
        assert torch.equal(out, expected)


@pytest.mark.gpu
def test_noalloc_matches_whisper_golden(dev):
    """The reference's own mel gate (max |d| <= 1e-3, mean |d| <= 1e-5
    against transformers' WhisperFeatureExtractor) on its full-chunk test
    signal, through the no-alloc entry point."""
    import torch

    lib = vlasr.load()
    stream = torch.cuda.current_stream(dev).cuda_stream
    g = np.load(GOLDEN / "mel_whisper.npz")
    pcm = torch.from_numpy(tone_pcm(480000, seed=42).reshape(1, -1).astype(np.float32)).to(dev)
    out = torch.full((1, 128, 3000), float("nan"), device=dev)
    _noalloc(lib, pcm, out, stream)
    torch.cuda.synchronize()
    mel = out[0].cpu().numpy()
    diff = np.abs(mel[:, g["full_frames"]].astype(np.float64) - g["full_subset"])
    assert diff.max() <= 1e-3 and diff.mean() <= 1e-5
