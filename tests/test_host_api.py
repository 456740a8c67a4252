"""CPU: the tensor-level wrapper refuses host tensors and bad shapes before
any library call (there is no CPU path), and the synthetic generators are
deterministic."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import vlasr
from vlasr import synth


def test_cpu_tensors_are_rejected():
    x = torch.zeros(4, 8, dtype=torch.bfloat16)
    w = torch.ones(8, dtype=torch.bfloat16)
    with pytest.raises(vlasr.VlasrInputError, match="CUDA"):
        vlasr.add_layernorm(x, None, w, None)
    with pytest.raises(vlasr.VlasrInputError, match="CUDA"):
        vlasr.add_rmsnorm(x, x, w)
    with pytest.raises(vlasr.VlasrInputError, match="CUDA"):
        vlasr.gelu_erf(x)
    with pytest.raises(vlasr.VlasrInputError, match="CUDA"):
        vlasr.swiglu(x, x)
    with pytest.raises(vlasr.VlasrInputError, match="CUDA"):
        vlasr.rope_(x.view(4, 1, 8), None, head_dim=8)
    with pytest.raises(vlasr.VlasrInputError, match="CUDA"):
        vlasr.logmel(torch.zeros(480000))
    with pytest.raises(vlasr.VlasrInputError, match="CUDA"):
        vlasr.embed_gather(torch.zeros(4, dtype=torch.int64), x)
    with pytest.raises(vlasr.VlasrInputError, match="CUDA"):
        vlasr.kv_append(x, x, x, x, torch.zeros(4, dtype=torch.int64))


def test_synthetic_audio_is_seeded_and_bounded():
    a = synth.audio_chunks(2, seed=3)
    b = synth.audio_chunks(2, seed=3)
    assert a.shape == (2, 480000) and a.dtype == np.float32
    np.testing.assert_array_equal(a, b)
    assert not np.array_equal(a[0], a[1])
    assert np.abs(a).max() <= 1.0


def test_pad_chunk_matches_reference_contract():
    x = synth.tone_pcm(1000)
    y = synth.pad_chunk(x)
    assert y.shape == (480000,) and np.array_equal(y[:1000], x) and not y[1000:].any()
    with pytest.raises(ValueError):
        synth.pad_chunk(np.zeros(480001, np.float32))


def test_chain_launch_count_matches_the_mel_batching():
    """gpu_launches in the bench line: per step a tile and a normalise launch
    per mel batch of at most 64 chunks, plus add+LN and GELU per layer."""
    from vlasr.pipeline import MEL_BATCH_CHUNKS, ChainShape, EncoderNormChain

    class _Shape:
        pass

    chain = _Shape()
    for chunks, groups, want in ((256, 1, 2 * 4 + 64), (65, 1, 2 * 2 + 64), (64, 1, 2 + 64),
                                 (32, 4, 2 * 4 + 64 * 4)):
        chain.shape = ChainShape(chunks=chunks)
        assert EncoderNormChain.launches_per_step(chain, groups) == want
    import re
    from pathlib import Path
    src = (Path(__file__).resolve().parents[1] / "videolingo-user_b200" / "csrc" /
           "vl_mel.cu").read_text()
    assert int(re.search(r"kBatchChunks = (\d+);", src).group(1)) == MEL_BATCH_CHUNKS
