"""CPU: the encoder oracle against transformers' GLM-ASR modules, and the
checkpoint reader/writer with the reference loader's validation rules
(VideoLingo-user native/asr/src/model_loader.cu:484-546, 629-754)."""

from __future__ import annotations

import json

import numpy as np
import pytest
import torch

import vlasr
from helpers import normwise
from oracle.encoder_ref import encode_fp32, rope_tables
from vlasr.checkpoint import (AsrModelConfig, expected_tensors, inspect_checkpoint, load_weights,
                              read_safetensors_header, write_checkpoint)
from vlasr.synth import synthetic_weights, write_synthetic_checkpoint

TINY = AsrModelConfig(audio_hidden=64, audio_intermediate=256, audio_layers=2, audio_heads=4,
                      audio_head_dim=16, audio_mel_bins=8, text_hidden=32, text_intermediate=48,
                      text_layers=1, text_heads=2, text_kv_heads=1, text_head_dim=16,
                      vocab_size=10, projector_mid=64)


def _torch_weights(cfg, seed=0):
    bits = synthetic_weights(cfg, seed)
    return {k: torch.from_numpy(v.view(np.int16)).view(torch.bfloat16) for k, v in bits.items()}


def _hf_modules(cfg, weights):
    from transformers.models.glmasr.configuration_glmasr import GlmAsrConfig, GlmAsrEncoderConfig
    from transformers.models.glmasr.modeling_glmasr import (GlmAsrEncoder,
                                                            GlmAsrMultiModalProjector)
    enc_cfg = GlmAsrEncoderConfig(hidden_size=cfg.audio_hidden,
                                  intermediate_size=cfg.audio_intermediate,
                                  num_hidden_layers=cfg.audio_layers,
                                  num_attention_heads=cfg.audio_heads,
                                  num_mel_bins=cfg.audio_mel_bins, max_position_embeddings=64)
    enc_cfg._attn_implementation = "eager"
    full = GlmAsrConfig(audio_config=enc_cfg.to_dict(),
                        text_config={"hidden_size": cfg.text_hidden,
                                     "intermediate_size": cfg.text_intermediate,
                                     "num_hidden_layers": 1, "num_attention_heads": cfg.text_heads,
                                     "num_key_value_heads": cfg.text_kv_heads,
                                     "vocab_size": cfg.vocab_size})
    enc = GlmAsrEncoder(enc_cfg).float().eval()
    proj = GlmAsrMultiModalProjector(full).float().eval()
    f32 = {k: v.float() for k, v in weights.items()}
    enc.load_state_dict({k[len("audio_tower."):]: v for k, v in f32.items()
                         if k.startswith("audio_tower.")}, strict=True)
    proj.load_state_dict({k[len("multi_modal_projector."):]: v for k, v in f32.items()
                          if k.startswith("multi_modal_projector.")}, strict=True)
    return enc, proj


def test_encoder_oracle_matches_transformers():
    w = _torch_weights(TINY, seed=1)
    enc, proj = _hf_modules(TINY, w)
    g = torch.Generator().manual_seed(2)
    mel = torch.rand(3, TINY.audio_mel_bins, 48, generator=g) * 2.5 - 1.0   # log-mel range
    with torch.no_grad():
        hs = enc(mel).last_hidden_state                                      # [3, 24, 64]
        ref = proj(hs.reshape(3, -1, TINY.audio_intermediate)).reshape(-1, TINY.text_hidden)
    got = encode_fp32(mel, w, heads=TINY.audio_heads, stages=True)
    assert normwise(got["final_norm"].numpy(), hs.reshape(-1, TINY.audio_hidden).numpy()) < 1e-5
    assert normwise(got["projector"].numpy(), ref.numpy()) < 1e-5


def test_rope_tables_follow_the_reference_recipe():
    cos, sin = rope_tables(1500, 32)
    i, d = 1234, 21
    ang = i / 10000.0 ** (((d % 16) * 2) / 32)
    assert cos[i, d].item() == np.float32(np.cos(ang))
    assert sin[i, d].item() == np.float32(np.sin(ang))


def test_checkpoint_round_trip(tmp_path):
    write_synthetic_checkpoint(tmp_path, TINY, seed=3)
    cfg, w = load_weights(tmp_path, "cpu")
    assert cfg == TINY
    assert set(w) == {n for n, _ in expected_tensors(TINY)}
    bits = synthetic_weights(TINY, 3)
    for name, t in w.items():
        assert t.dtype == torch.bfloat16 and t.shape == bits[name].shape
        assert np.array_equal(t.view(torch.int16).numpy().view(np.uint16), bits[name])
        assert t.data_ptr() % 256 == 0              # aligned arena slots
    _, sub = load_weights(tmp_path, "cpu", dtype=torch.float16, prefixes=("audio_tower.",))
    assert all(k.startswith("audio_tower.") for k in sub)
    assert sub["audio_tower.conv1.bias"].dtype == torch.float16
    # the same values as an independent safetensors reader
    from safetensors.torch import load_file
    ref = load_file(str(tmp_path / "model.safetensors"))
    assert all(torch.equal(ref[k], w[k]) for k in ref)


def test_subset_weights_match_full_set():
    full = synthetic_weights(TINY, 4)
    sub = synthetic_weights(TINY, 4, prefixes=("multi_modal_projector.",))
    assert sub and all(np.array_equal(full[k], sub[k]) for k in sub)


def _tensors(cfg):
    return synthetic_weights(cfg, 5)


def test_inventory_rejects_missing_unexpected_and_misshaped(tmp_path):
    t = _tensors(TINY)
    del t["audio_tower.layers.1.mlp.fc2.bias"]
    t["audio_tower.layers.0.self_attn.k_proj.bias"] = np.zeros(64, np.uint16)
    t["audio_tower.norm.weight"] = np.zeros(65, np.uint16)
    write_checkpoint(tmp_path, TINY, t)
    with pytest.raises(vlasr.VlasrInputError) as e:
        inspect_checkpoint(tmp_path)
    rep = json.loads(str(e.value).split(": ", 1)[1])
    assert rep["missing_tensors"] == ["audio_tower.layers.1.mlp.fc2.bias"]
    assert rep["unexpected_tensors"] == ["audio_tower.layers.0.self_attn.k_proj.bias"]
    assert rep["shape_mismatches"] == ["audio_tower.norm.weight: expected [64] got [65]"]


def test_projector_width_is_checked_for_consistency(tmp_path):
    t = _tensors(TINY)
    t["multi_modal_projector.linear_2.weight"] = np.zeros((32, 60), np.uint16)
    write_checkpoint(tmp_path, TINY, t)
    with pytest.raises(vlasr.VlasrInputError, match="linear_2.weight: expected \\[32, 64\\]"):
        inspect_checkpoint(tmp_path)


def _raw_file(path, header: dict, data: bytes = b"", header_size: int | None = None):
    raw = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write((len(raw) if header_size is None else header_size).to_bytes(8, "little"))
        f.write(raw)
        f.write(data)


@pytest.mark.parametrize("header,data,needle", [
    ({"a": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]}}, b"\0" * 8, "unsupported dtype"),
    ({"a": {"dtype": "BF16", "shape": [2], "data_offsets": [0, 8]}}, b"\0" * 4, "out of range"),
    ({"a": {"dtype": "BF16", "shape": [3], "data_offsets": [0, 4]}}, b"\0" * 4, "byte length"),
    ({"a": {"dtype": "BF16", "shape": [0], "data_offsets": [0, 0]}}, b"", "bad shape dim"),
    ({"a": {"dtype": "BF16", "shape": [2]}}, b"\0" * 4, "data_offsets"),
    ({"a": [1, 2]}, b"", "not an object"),
    ({"__metadata__": {"x": "y"}}, b"", "no tensors"),
])
def test_header_rules(tmp_path, header, data, needle):
    p = tmp_path / "model.safetensors"
    _raw_file(p, header, data)
    with pytest.raises(vlasr.VlasrInputError, match=needle):
        read_safetensors_header(p)


def test_header_size_and_missing_file(tmp_path):
    p = tmp_path / "model.safetensors"
    _raw_file(p, {}, header_size=0)
    with pytest.raises(vlasr.VlasrInputError, match="implausible"):
        read_safetensors_header(p)
    with pytest.raises(vlasr.VlasrInputError, match="cannot open"):
        read_safetensors_header(tmp_path / "absent.safetensors")


def test_config_rules(tmp_path):
    (tmp_path / "config.json").write_text(json.dumps({"audio_config": {}}))
    with pytest.raises(vlasr.VlasrInputError, match="text_config|hidden_size"):
        inspect_checkpoint(tmp_path)
    bad = TINY.to_json()
    bad["audio_config"]["head_dim"] = 15
    (tmp_path / "config.json").write_text(json.dumps(bad))
    with pytest.raises(vlasr.VlasrInputError, match="heads \\* head_dim"):
        inspect_checkpoint(tmp_path)


def test_audio_encoder_needs_cuda_weights():
    from vlasr.encoder import AudioEncoder
    w = _torch_weights(TINY, 6)
    with pytest.raises(vlasr.VlasrInputError, match="CUDA"):
        AudioEncoder(w, heads=TINY.audio_heads)
