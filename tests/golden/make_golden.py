"""Generate the golden vectors under tests/golden/ (committed with this script).

mel_whisper.npz
    transformers.WhisperFeatureExtractor(feature_size=128, sampling_rate=16000,
    hop_length=160, n_fft=400, chunk_length=30, dither=0.0) on the reference's
    own mel test signals - a full 30 s chunk (seed 42) and a 30000-sample clip
    zero-padded to 30 s (seed 7) - exactly as VideoLingo-user's
    tests/test_native_asr_m0.py:143-198 calls it.  That extractor is both the
    reference's production CPU mel path (pipeline/asr/glm.py:165-182) and its
    mel test oracle.  Stored: the full short-clip features, and frames
    [0,96) + [1452,1548) + [2904,3000) of the full chunk plus its global max
    and mean (the whole array is 1.5 MB).

ops_hf.npz
    fp32 outputs of the transformers GLM-ASR modeling semantics on small
    seeded inputs: nn.LayerNorm (encoder), Llama-style RMSNorm, exact GELU,
    silu(gate)*up, and rotate-half RoPE through transformers'
    modeling_glmasr.apply_rotary_pos_emb (encoder: rotary 32 of 64; decoder
    config: rotary 64 of 128).

Run from the repo root:  python tests/golden/make_golden.py
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent / "videolingo-user_b200"))

from vlasr.synth import pad_chunk, tone_pcm  # noqa: E402

MEL_FRAMES_KEPT = np.r_[0:96, 1452:1548, 2904:3000]


def whisper_mel(pcm32: np.ndarray) -> np.ndarray:
    from transformers import WhisperFeatureExtractor

    extractor = WhisperFeatureExtractor(feature_size=128, sampling_rate=16000, hop_length=160,
                                        n_fft=400, chunk_length=30, dither=0.0)
    return extractor(pcm32, sampling_rate=16000, truncation=False, padding="max_length",
                     return_tensors="np").input_features[0].astype(np.float32)


def make_mel() -> None:
    full = whisper_mel(tone_pcm(480000, seed=42))
    short = whisper_mel(tone_pcm(30000, seed=7))
    np.savez_compressed(HERE / "mel_whisper.npz",
                        full_frames=MEL_FRAMES_KEPT.astype(np.int32),
                        full_subset=full[:, MEL_FRAMES_KEPT],
                        full_max=np.float32(full.max()), full_mean=np.float64(full.mean()),
                        short=short)


def rope_hf(q: np.ndarray, k: np.ndarray, positions: np.ndarray, rotary_dim: int, base: float):
    """q/k [tokens, heads, head_dim]; transformers' fp32 cos/sin + apply_rotary_pos_emb."""
    from transformers.models.glmasr.modeling_glmasr import apply_rotary_pos_emb

    inv_freq = 1.0 / (base ** (torch.arange(0, rotary_dim, 2, dtype=torch.int64).float() / rotary_dim))
    pos = torch.from_numpy(positions.astype(np.float32))
    freqs = pos[:, None] * inv_freq[None, :]
    emb = torch.cat((freqs, freqs), dim=-1)
    cos, sin = emb.cos(), emb.sin()                 # [tokens, rotary_dim]
    qt = torch.from_numpy(q).transpose(0, 1)[None]  # [1, heads, tokens, hd]
    kt = torch.from_numpy(k).transpose(0, 1)[None]
    qe, ke = apply_rotary_pos_emb(qt, kt, cos[None], sin[None])
    return qe[0].transpose(0, 1).contiguous().numpy(), ke[0].transpose(0, 1).contiguous().numpy()


def make_ops() -> None:
    rng = np.random.default_rng(2024)
    f = lambda *s, m=0.0, sd=1.0: rng.normal(m, sd, size=s).astype(np.float32)  # noqa: E731
    d = {}
    # encoder add + LayerNorm
    d["ln_res"], d["ln_delta"] = f(4, 1280), f(4, 1280)
    d["ln_gamma"], d["ln_beta"] = f(1280, m=1.0, sd=0.02), f(1280, sd=0.02)
    h = torch.from_numpy(d["ln_res"] + d["ln_delta"])
    d["ln_out"] = F.layer_norm(h, (1280,), torch.from_numpy(d["ln_gamma"]),
                               torch.from_numpy(d["ln_beta"]), 1e-5).numpy()
    # decoder add + RMSNorm (Llama-style, fp32)
    d["rms_res"], d["rms_delta"] = f(4, 2048), f(4, 2048)
    d["rms_w"] = f(2048, m=1.0, sd=0.02)
    h = torch.from_numpy(d["rms_res"] + d["rms_delta"])
    var = h.pow(2).mean(-1, keepdim=True)
    d["rms_out"] = (h * torch.rsqrt(var + 1e-5) * torch.from_numpy(d["rms_w"])).numpy()
    # GELU (erf) and SwiGLU
    d["gelu_in"] = f(2, 2048, sd=3.0)
    d["gelu_out"] = F.gelu(torch.from_numpy(d["gelu_in"])).numpy()
    d["swi_g"], d["swi_u"] = f(2, 2048, sd=3.0), f(2, 2048)
    d["swi_out"] = (F.silu(torch.from_numpy(d["swi_g"])) * torch.from_numpy(d["swi_u"])).numpy()
    # encoder RoPE: 20 heads x 64, rotary 32, positions = frame index
    d["rope_enc_q"], d["rope_enc_k"] = f(12, 20, 64), f(12, 20, 64)
    d["rope_enc_pos"] = np.array([0, 1, 2, 3, 100, 511, 512, 777, 1000, 1234, 1498, 1499], np.int64)
    d["rope_enc_q_out"], d["rope_enc_k_out"] = rope_hf(d["rope_enc_q"], d["rope_enc_k"],
                                                       d["rope_enc_pos"], 32, 10000.0)
    # decoder config: 16 q / 4 k heads x 128, rotary 64 (first half)
    d["rope_dec_q"], d["rope_dec_k"] = f(8, 16, 128), f(8, 4, 128)
    d["rope_dec_pos"] = np.array([0, 1, 7, 63, 64, 1023, 2047, 4095], np.int64)
    d["rope_dec_q_out"], d["rope_dec_k_out"] = rope_hf(d["rope_dec_q"], d["rope_dec_k"],
                                                       d["rope_dec_pos"], 64, 10000.0)
    np.savez_compressed(HERE / "ops_hf.npz", **d)


if __name__ == "__main__":
    make_mel()
    make_ops()
    for p in sorted(HERE.glob("*.npz")):
        print(p.name, p.stat().st_size)
