"""The reference's own CPU implementation of the hot path, for the bench's
CPU baseline and the `--impl reference` arm.  TEST/BASELINE INFRASTRUCTURE
ONLY (never part of the product path).

VideoLingo-user runs GLM-ASR on the CPU through transformers
(pipeline/asr/glm.py:165-182): the processor's WhisperFeatureExtractor
computes the log-mel features, and the GlmAsr encoder layers apply
nn.LayerNorm after the residual add and exact-erf GELU in the MLP
(transformers models/glmasr/modeling_glmasr.py, GlmAsrEncoderLayer /
GlmAsrMLP).  This module calls exactly those: the extractor with the
reference's parameters and torch's CPU layer_norm / gelu in bf16, with all
host threads torch is allowed to use.
"""

from __future__ import annotations

import os
import time

import numpy as np


def whisper_extractor():
    from transformers import WhisperFeatureExtractor
    return WhisperFeatureExtractor(feature_size=128, sampling_rate=16000, hop_length=160,
                                   n_fft=400, chunk_length=30, dither=0.0)


def mel_features(extractor, pcm: np.ndarray) -> np.ndarray:
    """[chunks, 480000] f32 -> [chunks, 128, 3000] via WhisperFeatureExtractor."""
    return extractor(list(pcm), sampling_rate=16000, truncation=False, padding="max_length",
                     return_tensors="np").input_features


def encoder_chain(h, y, g_in, gammas, betas):
    """layers x (h = h + y; y = LayerNorm(h); GELU(g_in)) in bf16 on the CPU."""
    import torch
    import torch.nn.functional as F
    out = None
    for l in range(gammas.shape[0]):
        h = h + y
        y = F.layer_norm(h, (h.shape[-1],), gammas[l], betas[l], 1e-5)
        out = F.gelu(g_in)
    return h, y, out


def time_sample(chunks: int, layers: int = 32, seed: int = 0, threads: int | None = None) -> dict:
    """Run `chunks` chunks of the box-scale chain on the CPU; returns timings."""
    import torch
    from vlasr.synth import audio_chunks

    threads = threads or os.cpu_count() or 1
    torch.set_num_threads(threads)
    pcm = audio_chunks(chunks, seed=seed)
    g = torch.Generator().manual_seed(seed)
    bf = torch.bfloat16
    rows = chunks * 1500
    h = torch.randn(rows, 1280, generator=g).to(bf)
    y = torch.randn(rows, 1280, generator=g).to(bf)
    g_in = torch.randn(rows, 5120, generator=g).to(bf)
    gammas = (1.0 + 0.02 * torch.randn(layers, 1280, generator=g)).to(bf)
    betas = (0.02 * torch.randn(layers, 1280, generator=g)).to(bf)
    fe = whisper_extractor()
    t0 = time.perf_counter()
    mel_features(fe, pcm)
    t1 = time.perf_counter()
    encoder_chain(h, y, g_in, gammas, betas)
    t2 = time.perf_counter()
    return {"chunks": chunks, "layers": layers, "threads": threads, "mel_s": t1 - t0,
            "layers_s": t2 - t1, "total_s": t2 - t0}
