"""GPU parity of the log-mel frontend.

* against transformers' WhisperFeatureExtractor golden vectors with the
  reference's own gate (max abs <= 1e-3, mean abs <= 1e-5;
  VideoLingo-user tests/test_native_asr_m0.py:174-198), on the reference's
  test signals (full chunk seed 42; 30000-sample clip seed 7, zero-padded);
* against the float64 oracle: normwise relative error <= 1e-5 (fp32);
* per-chunk independence across the kernel's batch boundary (32 chunks);
* silence, clipping-level input and invalid arguments.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
import vlasr
from conftest import GOLDEN
from helpers import normwise, to_np
from vlasr.synth import audio_chunks, pad_chunk, tone_pcm

pytestmark = pytest.mark.gpu


def _mel(dev, pcm: np.ndarray) -> np.ndarray:
    x = torch.from_numpy(np.ascontiguousarray(pcm, np.float32).reshape(-1, 480000)).to(dev)
    return to_np(vlasr.logmel(x))


def _gate(produced, reference, max_abs=1e-3, mean_abs=1e-5):
    diff = np.abs(np.asarray(produced, np.float64) - np.asarray(reference, np.float64))
    assert diff.max() <= max_abs, diff.max()
    assert diff.mean() <= mean_abs, diff.mean()
    return diff.max()


def test_full_chunk_matches_whisper_golden(dev):
    g = np.load(GOLDEN / "mel_whisper.npz")
    mel = _mel(dev, tone_pcm(480000, seed=42))[0]
    _gate(mel[:, g["full_frames"]], g["full_subset"])
    assert abs(float(mel.max()) - float(g["full_max"])) <= 1e-4
    assert abs(float(mel.mean()) - float(g["full_mean"])) <= 1e-5


def test_short_clip_zero_padding_matches_whisper_golden(dev):
    g = np.load(GOLDEN / "mel_whisper.npz")
    mel = _mel(dev, pad_chunk(tone_pcm(30000, seed=7)))[0]
    _gate(mel, g["short"])


def test_matches_float64_oracle_normwise(dev):
    pcm = audio_chunks(2, seed=5)
    mel = _mel(dev, pcm)
    exp = oracle.logmel_f64(pcm)
    assert normwise(mel, exp) <= 1e-5
    _gate(mel, exp, max_abs=2e-4, mean_abs=2e-6)


def test_matches_reference_fp32_restatement(dev):
    pcm = audio_chunks(1, seed=9)
    _gate(_mel(dev, pcm), oracle.logmel_ref(pcm), max_abs=2e-4, mean_abs=2e-6)


def test_chunks_are_independent_across_batches(dev):
    """67 chunks span two kernel batches (33 + 34); each chunk equals its own
    1-chunk run."""
    pcm = audio_chunks(67, seed=13)
    pcm[4] *= 0.01           # different chunk maxima
    pcm[35] = 0.0            # silent chunk in the second batch
    many = _mel(dev, pcm)
    for c in (0, 4, 32, 33, 35, 66):
        one = _mel(dev, pcm[c])
        np.testing.assert_array_equal(many[c], one[0])
    exp = oracle.logmel_f64(pcm[[0, 33, 66]])
    assert normwise(many[[0, 33, 66]], exp) <= 1e-5


def test_silence_and_full_scale(dev):
    pcm = np.zeros((2, 480000), np.float32)
    pcm[1] = np.sign(np.sin(np.arange(480000) * 0.3)).astype(np.float32)  # full-scale square
    mel = _mel(dev, pcm)
    # silence: log10(1e-10) = -10 everywhere, clamp is a no-op, (x+4)/4 = -1.5
    np.testing.assert_array_equal(mel[0], np.full((128, 3000), -1.5, np.float32))
    assert normwise(mel[1], oracle.logmel_f64(pcm[1])[0]) <= 1e-5


def test_reflect_padding_edges(dev):
    """Energy only in the first/last 200 samples exercises the reflect pad."""
    pcm = np.zeros(480000, np.float32)
    rng = np.random.default_rng(3)
    pcm[:300] = rng.normal(0, 0.5, 300)
    pcm[-300:] = rng.normal(0, 0.5, 300)
    mel = _mel(dev, pcm)
    exp = oracle.logmel_f64(pcm)
    _gate(mel[0][:, :4], exp[0][:, :4], max_abs=2e-4)
    _gate(mel[0][:, -4:], exp[0][:, -4:], max_abs=2e-4)


def test_repeatable_and_workspace_reuse(dev):
    pcm = torch.from_numpy(audio_chunks(3, seed=1)).to(dev)
    ws = torch.empty(vlasr.logmel_workspace_bytes(3), dtype=torch.uint8, device=dev)
    out = torch.empty(3, 128, 3000, device=dev)
    a = vlasr.logmel(pcm, out=out, workspace=ws).clone()
    ws.fill_(0xFF)  # garbage workspace must not matter
    b = vlasr.logmel(pcm, out=out, workspace=ws)
    assert torch.equal(a, b)


def test_invalid_inputs(dev):
    with pytest.raises(vlasr.VlasrInputError):
        vlasr.logmel(torch.zeros(480001, device=dev))
    with pytest.raises(vlasr.VlasrInputError):
        vlasr.logmel(torch.zeros(480000, device=dev, dtype=torch.float16))
    x = torch.zeros(480000, device=dev)
    with pytest.raises(vlasr.VlasrInputError, match="workspace"):
        vlasr.logmel(x, workspace=torch.empty(8, dtype=torch.uint8, device=dev))
    with pytest.raises(vlasr.VlasrInputError, match="aligned"):
        buf = torch.zeros(480001, device=dev)
        vlasr.logmel(buf[1:])
