"""Seeded synthetic inputs with the shapes and value distributions of the
benchmark configurations (no real audio or checkpoint is needed).

* audio chunks: 30 s of 16 kHz mono f32 = sum of 8 sinusoids (frequency
  U(80, 4000) Hz, amplitude U(0, 0.1), phase U(0, 2pi)) + N(0, 0.01) noise,
  clipped to [-1, 1]; one independent seed per chunk.
* activations N(0, 1), LayerNorm gamma N(1, 0.02), beta N(0, 0.02), RMSNorm
  weight N(1, 0.02), embedding table N(0, 0.02), token ids U[0, vocab).

The reference's own mel test signal (three sines plus 0.05*N(0,1),
tests/test_native_asr_m0.py:143-154 of VideoLingo-user) is `tone_pcm`.
"""

from __future__ import annotations

import numpy as np

SAMPLE_RATE = 16000
CHUNK_SAMPLES = 480000


def audio_chunk(seed: int, samples: int = CHUNK_SAMPLES) -> np.ndarray:
    rng = np.random.default_rng(seed)
    freqs = rng.uniform(80.0, 4000.0, size=8)
    amps = rng.uniform(0.0, 0.1, size=8)
    phases = rng.uniform(0.0, 2.0 * np.pi, size=8)
    t = np.arange(samples, dtype=np.float64) / SAMPLE_RATE
    x = (amps[:, None] * np.sin(2.0 * np.pi * freqs[:, None] * t[None, :] + phases[:, None])).sum(0)
    x += rng.normal(0.0, 0.01, size=samples)
    return np.clip(x, -1.0, 1.0).astype(np.float32)


def audio_chunks(chunks: int, seed: int = 0, samples: int = CHUNK_SAMPLES) -> np.ndarray:
    """[chunks, samples] f32, chunk c seeded with seed*100003 + c."""
    out = np.empty((chunks, samples), dtype=np.float32)
    for c in range(chunks):
        out[c] = audio_chunk(seed * 100003 + c, samples)
    return out


def tone_pcm(sample_count: int, seed: int = 42) -> np.ndarray:
    """440/1234/3000 Hz sines + 0.05*N(0,1) (the reference mel test signal)."""
    rng = np.random.default_rng(seed)
    t = np.arange(sample_count, dtype=np.float64)
    signal = (0.3 * np.sin(2 * np.pi * 440 * t / 16000)
              + 0.2 * np.sin(2 * np.pi * 1234 * t / 16000)
              + 0.1 * np.sin(2 * np.pi * 3000 * t / 16000)
              + 0.05 * rng.standard_normal(sample_count))
    return signal.astype(np.float32)


def pad_chunk(pcm: np.ndarray) -> np.ndarray:
    """Zero-pad (or reject) a clip to one 30 s chunk, as the reference CLI does
    (native/asr/src/main_m0.cu:60-79)."""
    if pcm.size > CHUNK_SAMPLES:
        raise ValueError("PCM exceeds the 30 s chunk (480000 samples)")
    out = np.zeros(CHUNK_SAMPLES, dtype=np.float32)
    out[:pcm.size] = pcm
    return out


def normal(shape, seed: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return rng.normal(mean, std, size=shape).astype(np.float32)


def audio_chunks_device(chunks: int, first_chunk: int, seed: int, device):
    """[chunks, 480000] f32 torch tensor on `device` with the audio_chunk
    recipe: sinusoid parameters drawn per chunk from numpy exactly as
    audio_chunk does, the sum evaluated in fp64 on the device, and
    N(0, 0.01) noise from a seeded torch generator (fast for hundreds of
    chunks; the noise differs from audio_chunk's numpy stream)."""
    import torch
    params = np.empty((chunks, 3, 8), dtype=np.float64)
    for i in range(chunks):
        rng = np.random.default_rng(seed * 100003 + first_chunk + i)
        params[i, 0] = rng.uniform(80.0, 4000.0, size=8)
        params[i, 1] = rng.uniform(0.0, 0.1, size=8)
        params[i, 2] = rng.uniform(0.0, 2.0 * np.pi, size=8)
    p = torch.from_numpy(params).to(device)
    t = torch.arange(CHUNK_SAMPLES, device=device, dtype=torch.float64) / SAMPLE_RATE
    out = torch.empty((chunks, CHUNK_SAMPLES), device=device, dtype=torch.float32)
    gen = torch.Generator(device=device)
    gen.manual_seed(seed * 100003 + first_chunk)
    for i in range(chunks):
        x = (p[i, 1, :, None] * torch.sin(2.0 * np.pi * p[i, 0, :, None] * t[None, :]
                                          + p[i, 2, :, None])).sum(0)
        noise = torch.empty(CHUNK_SAMPLES, device=device, dtype=torch.float64)
        noise.normal_(0.0, 0.01, generator=gen)
        out[i] = (x + noise).clamp_(-1.0, 1.0).float()
    return out


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """f32 -> BF16 bit patterns (uint16) by truncation (the high half of each
    little-endian f32)."""
    return np.ascontiguousarray(np.ascontiguousarray(x, dtype=np.float32).view(np.uint16)[..., 1::2])


def synthetic_weights(cfg, seed: int = 0, prefixes=None) -> dict:
    """Seeded BF16 bit patterns for every tensor of the official GLM-ASR
    inventory of `cfg` (an AsrModelConfig), drawn uniformly with the standard
    deviations of a usual initialisation: matrices and conv kernels
    1/sqrt(fan_in), biases and embeddings 0.02, norm weights 1 +- 0.02, norm
    biases 0.02.  Tensor i draws from the generator seeded with [seed, i], so
    a subset (`prefixes`) has the same values as the full set."""
    from .checkpoint import expected_tensors
    out = {}
    half_width = np.float32(np.sqrt(3.0))       # U(-a, a) has std a / sqrt(3)
    for i, (name, shape) in enumerate(expected_tensors(cfg)):
        if prefixes is not None and not name.startswith(tuple(prefixes)):
            continue
        rng = np.random.default_rng([seed, i])
        x = rng.random(shape, dtype=np.float32)
        x *= 2.0 * half_width
        x -= half_width                           # unit variance
        if "norm" in name and name.endswith(".weight"):
            x *= np.float32(0.02)
            x += np.float32(1.0)
        elif name.endswith(".bias") or "embed_tokens" in name:
            x *= np.float32(0.02)
        else:
            x *= np.float32(1.0 / np.sqrt(int(np.prod(shape[1:]))))
        out[name] = bf16_bits(x)
    return out


def write_synthetic_checkpoint(model_dir, cfg=None, seed: int = 0):
    """config.json + model.safetensors with synthetic_weights(cfg, seed).

    The default config is GLM-ASR-Nano's audio tower and projector with a
    one-layer, 64-token text model: the full official inventory (the
    reference's loader accepts it), ~1.4 GB instead of ~4.5 GB."""
    from .checkpoint import AsrModelConfig, write_checkpoint
    if cfg is None:
        cfg = AsrModelConfig(text_layers=1, vocab_size=64)
    write_checkpoint(model_dir, cfg, synthetic_weights(cfg, seed))
    return cfg
