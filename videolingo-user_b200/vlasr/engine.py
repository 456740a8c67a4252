"""In-process GLM-ASR engine: PCM chunks -> log-mel -> audio tower + projector
-> text decoder -> generated token ids per chunk.

The in-process counterpart of the reference engine's `transcribe` command
(VideoLingo-user native/asr/src/main_m0.cu:440-490, driven by
pipeline/asr/native.py:119-276 through a subprocess): the same input
contract - mono 16 kHz f32 PCM cut into whole 30 s chunks, a shared prompt
of token ids, greedy decode up to a token budget - and the same output
(token ids per chunk, through the first EOS), with every stage resident on
one GPU and no host round trip between them.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import ops
from ._lib import VlasrInputError
from .checkpoint import load_weights
from .decoder import TextDecoder
from .encoder import AudioEncoder
from .synth import CHUNK_SAMPLES

MAX_CHUNKS = 128   # the reference engine's limit per call (native.py:155-157)


@dataclass
class EngineTimings:
    mel_ms: float = 0.0
    encode_ms: float = 0.0
    decode_ms: float = 0.0       # prefill + decode steps
    prefill_ms: float = 0.0
    steps_ms: float = 0.0


def pad_to_chunks(pcm: np.ndarray, chunk_samples: int = CHUNK_SAMPLES) -> np.ndarray:
    """Mono f32 PCM -> [chunks, chunk_samples], the tail padded with silence
    (pipeline/asr/native.py:150-164)."""
    pcm = np.asarray(pcm, dtype=np.float32).reshape(-1)
    if pcm.size == 0:
        raise VlasrInputError("decoded audio is empty")
    chunks = (pcm.size + chunk_samples - 1) // chunk_samples
    if chunks > MAX_CHUNKS:
        raise VlasrInputError(f"the engine supports 1..{MAX_CHUNKS} chunks, got {chunks}")
    out = np.zeros((chunks, chunk_samples), dtype=np.float32)
    out.reshape(-1)[:pcm.size] = pcm
    return out


class AsrEngine:
    """Resident GLM-ASR weights and the three stages.  Either from a
    checkpoint directory or from already loaded weights (name -> tensor)."""

    def __init__(self, model_dir=None, *, weights: dict | None = None, device="cuda:0",
                 dtype=torch.bfloat16, max_seq_len: int = 1024):
        self.device = torch.device(device)
        if weights is None:
            if model_dir is None:
                raise VlasrInputError("AsrEngine needs a model_dir or weights")
            cfg, weights = load_weights(model_dir, self.device)
            heads, text_heads, kv_heads = cfg.audio_heads, cfg.text_heads, cfg.text_kv_heads
        else:
            heads, text_heads, kv_heads = 20, 16, 4
        self.encoder = AudioEncoder(weights, heads=heads, dtype=dtype)
        self.decoder = TextDecoder(weights, heads=text_heads, kv_heads=kv_heads, dtype=dtype,
                                   max_seq_len=max_seq_len)
        self.timings = EngineTimings()

    def transcribe_ids(self, pcm, prompt_ids, max_new_tokens: int = 256) -> list[list[int]]:
        """pcm: [samples] or [chunks, 480000] f32 (numpy or torch, host or
        device) -> generated ids per chunk."""
        if isinstance(pcm, torch.Tensor) and pcm.dim() == 2:
            chunks_t = pcm.to(self.device, torch.float32).contiguous()
        else:
            arr = pcm.cpu().numpy() if isinstance(pcm, torch.Tensor) else np.asarray(pcm)
            chunks_np = arr if arr.ndim == 2 else pad_to_chunks(arr)
            if chunks_np.shape[1] != CHUNK_SAMPLES:
                raise VlasrInputError("chunks must hold 480000 samples each")
            if not 1 <= chunks_np.shape[0] <= MAX_CHUNKS:
                raise VlasrInputError(f"the engine supports 1..{MAX_CHUNKS} chunks")
            chunks_t = torch.from_numpy(np.ascontiguousarray(chunks_np, dtype=np.float32)).to(
                self.device, non_blocking=False)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        ev[0].record()
        mel = ops.logmel(chunks_t)
        ev[1].record()
        audio = self.encoder.encode(mel)
        ev[2].record()
        result = self.decoder.generate(audio, prompt_ids, max_new_tokens=max_new_tokens)
        ev[3].record()
        torch.cuda.synchronize(self.device)
        self.timings = EngineTimings(ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2]),
                                     ev[2].elapsed_time(ev[3]), *self.decoder.last_timings)
        return result.per_chunk_ids


def transcribe_ids_sharded(engine, pcm_chunks, prompt_ids, max_new_tokens: int = 256,
                           group=None) -> list[list[int]]:
    """Multi-GPU engine call: one process per GPU, chunks sharded by
    contiguous range over the ranks of `group` (the partition of the
    benchmark chain, vlasr.pipeline.shard_range); every rank runs its shard
    on its own engine and the id lists are all-gathered, so every rank
    returns the ids of all chunks in chunk order.  Chunks are independent
    (per-chunk mel normalisation, unmasked per-chunk encoder attention,
    per-chunk decode), so the ids equal a single-GPU call's."""
    import torch.distributed as dist
    from .pipeline import shard_range
    chunks_np = pcm_chunks if np.asarray(pcm_chunks).ndim == 2 else pad_to_chunks(pcm_chunks)
    chunks = chunks_np.shape[0]
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    c0, c1 = shard_range(chunks, rank, world)
    mine = engine.transcribe_ids(chunks_np[c0:c1], prompt_ids,
                                 max_new_tokens=max_new_tokens) if c1 > c0 else []
    gathered: list = [None] * world
    dist.all_gather_object(gathered, mine, group=group)
    out: list[list[int]] = []
    for part in gathered:
        out.extend(part)
    if len(out) != chunks:
        raise VlasrInputError(f"sharded engine returned {len(out)} transcripts for {chunks} chunks")
    return out
