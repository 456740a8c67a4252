"""GLM-ASR checkpoint reader: `config.json` + `model.safetensors` (BF16) ->
resident device tensors, after the official tensor-inventory check.

Follows the reference's loader (VideoLingo-user
native/asr/src/model_loader.cu):

* config keys `audio_config.*` / `text_config.*` and the heads x head_dim
  consistency checks (parse_model_config, :629-660);
* safetensors header rules (read_safetensors_header, :664-720): a header of
  1 B..64 MiB holding a JSON object; per tensor `dtype` "BF16" only, shape
  dims in (0, 2^30], `data_offsets` inside the data region, byte length =
  2 x elements;
* the expected inventory of GlmAsrForConditionalGeneration
  (expected_tensors, :484-546) and its check (validate_inventory, :722-754):
  missing, unexpected and mis-shaped tensors are listed, sorted, and any of
  them rejects the checkpoint.

Errors map onto the reference's taxonomy: a bad layout or argument raises
VlasrInputError (ModelInputError, CLI exit 2).

Unlike the reference (BF16 -> FP16 conversion through a staging buffer with
a device sync per tensor, :834-894), the kernels here compute in bf16, so the
tensors stay BF16: the data region is read once into pinned host memory and
each tensor is copied into a 256-byte aligned slot of one device arena.
`dtype=torch.float16` converts on the device afterwards (what the
reference's engine consumes).
"""

from __future__ import annotations

import json
import os
from dataclasses import dataclass, field, replace
from pathlib import Path

import numpy as np

from ._lib import VlasrInputError

MAX_HEADER_BYTES = 64 << 20
ARENA_ALIGN = 256


@dataclass(frozen=True)
class AsrModelConfig:
    """Model dimensions from config.json (official key names)."""
    audio_hidden: int = 1280
    audio_intermediate: int = 5120
    audio_layers: int = 32
    audio_heads: int = 20
    audio_head_dim: int = 64
    audio_mel_bins: int = 128
    text_hidden: int = 2048
    text_intermediate: int = 6144
    text_layers: int = 28
    text_heads: int = 16
    text_kv_heads: int = 4
    text_head_dim: int = 128
    vocab_size: int = 59264
    projector_mid: int = 4096   # not in config.json (the reference fixes it too)

    def to_json(self) -> dict:
        return {
            "audio_config": {
                "hidden_size": self.audio_hidden, "intermediate_size": self.audio_intermediate,
                "num_hidden_layers": self.audio_layers,
                "num_attention_heads": self.audio_heads, "head_dim": self.audio_head_dim,
                "num_mel_bins": self.audio_mel_bins},
            "text_config": {
                "hidden_size": self.text_hidden, "intermediate_size": self.text_intermediate,
                "num_hidden_layers": self.text_layers, "num_attention_heads": self.text_heads,
                "num_key_value_heads": self.text_kv_heads, "head_dim": self.text_head_dim,
                "vocab_size": self.vocab_size},
        }


def _require(obj: dict, key: str, where: str):
    if not isinstance(obj, dict) or key not in obj:
        raise VlasrInputError(f"missing key '{key}' in {where}")
    return obj[key]


def _require_int(obj: dict, key: str, where: str) -> int:
    v = _require(obj, key, where)
    if isinstance(v, bool) or not isinstance(v, (int, float)) or int(v) != v:
        raise VlasrInputError(f"expected integer for {where}.{key}")
    return int(v)


def parse_model_config(model_dir: str | os.PathLike) -> AsrModelConfig:
    """config.json -> AsrModelConfig (model_loader.cu:629-660)."""
    path = Path(model_dir) / "config.json"
    try:
        root = json.loads(path.read_text())
    except FileNotFoundError:
        raise VlasrInputError(f"cannot open {path}") from None
    except json.JSONDecodeError as e:
        raise VlasrInputError(f"config.json: {e}") from None
    if not isinstance(root, dict):
        raise VlasrInputError("config.json: expected object")
    a = _require(root, "audio_config", "config.json")
    t = _require(root, "text_config", "config.json")
    cfg = AsrModelConfig(
        audio_hidden=_require_int(a, "hidden_size", "audio_config"),
        audio_intermediate=_require_int(a, "intermediate_size", "audio_config"),
        audio_layers=_require_int(a, "num_hidden_layers", "audio_config"),
        audio_heads=_require_int(a, "num_attention_heads", "audio_config"),
        audio_head_dim=_require_int(a, "head_dim", "audio_config"),
        audio_mel_bins=_require_int(a, "num_mel_bins", "audio_config"),
        text_hidden=_require_int(t, "hidden_size", "text_config"),
        text_intermediate=_require_int(t, "intermediate_size", "text_config"),
        text_layers=_require_int(t, "num_hidden_layers", "text_config"),
        text_heads=_require_int(t, "num_attention_heads", "text_config"),
        text_kv_heads=_require_int(t, "num_key_value_heads", "text_config"),
        text_head_dim=_require_int(t, "head_dim", "text_config"),
        vocab_size=_require_int(t, "vocab_size", "text_config"),
    )
    if cfg.audio_heads * cfg.audio_head_dim != cfg.audio_hidden:
        raise VlasrInputError("audio_config: heads * head_dim != hidden_size")
    if cfg.text_heads * cfg.text_head_dim != cfg.text_hidden:
        raise VlasrInputError("text_config: heads * head_dim != hidden_size")
    return cfg


def expected_tensors(cfg: AsrModelConfig) -> list[tuple[str, tuple[int, ...]]]:
    """The official GlmAsrForConditionalGeneration inventory (model_loader.cu:484-546):
    Whisper-style audio tower (LayerNorm with bias; q/v/o biases, none on k),
    two-layer GELU projector with biases, Llama-style text model without biases."""
    ah, ai, mel = cfg.audio_hidden, cfg.audio_intermediate, cfg.audio_mel_bins
    th, ti = cfg.text_hidden, cfg.text_intermediate
    kv, vs = cfg.text_kv_heads * cfg.text_head_dim, cfg.vocab_size
    out: list[tuple[str, tuple[int, ...]]] = [
        ("audio_tower.conv1.weight", (ah, mel, 3)), ("audio_tower.conv1.bias", (ah,)),
        ("audio_tower.conv2.weight", (ah, ah, 3)), ("audio_tower.conv2.bias", (ah,)),
    ]
    for l in range(cfg.audio_layers):
        p = f"audio_tower.layers.{l}."
        out += [
            (p + "input_layernorm.weight", (ah,)), (p + "input_layernorm.bias", (ah,)),
            (p + "self_attn.q_proj.weight", (ah, ah)), (p + "self_attn.q_proj.bias", (ah,)),
            (p + "self_attn.k_proj.weight", (ah, ah)),
            (p + "self_attn.v_proj.weight", (ah, ah)), (p + "self_attn.v_proj.bias", (ah,)),
            (p + "self_attn.o_proj.weight", (ah, ah)), (p + "self_attn.o_proj.bias", (ah,)),
            (p + "post_attention_layernorm.weight", (ah,)),
            (p + "post_attention_layernorm.bias", (ah,)),
            (p + "mlp.fc1.weight", (ai, ah)), (p + "mlp.fc1.bias", (ai,)),
            (p + "mlp.fc2.weight", (ah, ai)), (p + "mlp.fc2.bias", (ah,)),
        ]
    out += [
        ("audio_tower.norm.weight", (ah,)), ("audio_tower.norm.bias", (ah,)),
        ("multi_modal_projector.linear_1.weight", (cfg.projector_mid, ah * 4)),
        ("multi_modal_projector.linear_1.bias", (cfg.projector_mid,)),
        ("multi_modal_projector.linear_2.weight", (th, cfg.projector_mid)),
        ("multi_modal_projector.linear_2.bias", (th,)),
        ("language_model.model.embed_tokens.weight", (vs, th)),
    ]
    for l in range(cfg.text_layers):
        p = f"language_model.model.layers.{l}."
        out += [
            (p + "input_layernorm.weight", (th,)),
            (p + "self_attn.q_proj.weight", (th, th)),
            (p + "self_attn.k_proj.weight", (kv, th)),
            (p + "self_attn.v_proj.weight", (kv, th)),
            (p + "self_attn.o_proj.weight", (th, th)),
            (p + "post_attention_layernorm.weight", (th,)),
            (p + "mlp.gate_proj.weight", (ti, th)),
            (p + "mlp.up_proj.weight", (ti, th)),
            (p + "mlp.down_proj.weight", (th, ti)),
        ]
    out += [("language_model.model.norm.weight", (th,)),
            ("language_model.lm_head.weight", (vs, th))]
    return out


@dataclass
class TensorSpec:
    name: str
    shape: tuple[int, ...]
    begin: int      # byte offsets within the data region
    end: int

    @property
    def nbytes(self) -> int:
        return self.end - self.begin

    @property
    def elements(self) -> int:
        n = 1
        for d in self.shape:
            n *= d
        return n


def read_safetensors_header(path: str | os.PathLike) -> tuple[list[TensorSpec], int]:
    """-> (tensors sorted by name, data region offset) (model_loader.cu:664-720)."""
    path = Path(path)
    try:
        size = path.stat().st_size
        with open(path, "rb") as f:
            head = f.read(8)
            if len(head) < 8:
                raise VlasrInputError(f"safetensors file too short: {path}")
            header_size = int.from_bytes(head, "little")
            if header_size == 0 or header_size > MAX_HEADER_BYTES:
                raise VlasrInputError(f"implausible safetensors header size: {header_size}")
            raw = f.read(header_size)
    except FileNotFoundError:
        raise VlasrInputError(f"cannot open safetensors file: {path}") from None
    if len(raw) != header_size:
        raise VlasrInputError("failed to read safetensors header")
    try:
        root = json.loads(raw)
    except (json.JSONDecodeError, UnicodeDecodeError) as e:
        raise VlasrInputError(f"safetensors header: {e}") from None
    if not isinstance(root, dict):
        raise VlasrInputError("safetensors header: expected object")
    data_offset = 8 + header_size
    data_size = size - data_offset
    tensors = []
    for name, spec in root.items():
        if name == "__metadata__":
            continue
        if not isinstance(spec, dict):
            raise VlasrInputError(f"safetensors header: tensor entry is not an object: {name}")
        dtype = _require(spec, "dtype", name)
        if not isinstance(dtype, str):
            raise VlasrInputError(f"bad dtype for {name}")
        shape = _require(spec, "shape", name)
        if not isinstance(shape, list):
            raise VlasrInputError(f"bad shape for {name}")
        dims = []
        for d in shape:
            if isinstance(d, bool) or not isinstance(d, int) or d <= 0 or d > (1 << 30):
                raise VlasrInputError(f"bad shape dim for {name}")
            dims.append(d)
        offs = _require(spec, "data_offsets", name)
        if (not isinstance(offs, list) or len(offs) != 2
                or not all(isinstance(o, int) and not isinstance(o, bool) and o >= 0
                           for o in offs)):
            raise VlasrInputError(f"bad data_offsets for {name}")
        t = TensorSpec(name, tuple(dims), offs[0], offs[1])
        if t.begin > t.end or t.end > data_size:
            raise VlasrInputError(f"data_offsets out of range for {name}")
        if dtype != "BF16":
            raise VlasrInputError(f"unsupported dtype {dtype} for {name}")
        if t.nbytes != 2 * t.elements:
            raise VlasrInputError(f"byte length mismatch for {name}")
        tensors.append(t)
    tensors.sort(key=lambda t: t.name)
    if not tensors:
        raise VlasrInputError("safetensors file contains no tensors")
    return tensors, data_offset


@dataclass
class InventoryReport:
    missing: list[str] = field(default_factory=list)
    unexpected: list[str] = field(default_factory=list)
    shape_mismatches: list[str] = field(default_factory=list)

    @property
    def ok(self) -> bool:
        return not (self.missing or self.unexpected or self.shape_mismatches)

    def to_json(self) -> dict:
        return {"missing_tensors": self.missing, "unexpected_tensors": self.unexpected,
                "shape_mismatches": self.shape_mismatches}


def validate_inventory(tensors: list[TensorSpec], cfg: AsrModelConfig) -> InventoryReport:
    """Compare a header against the official inventory (model_loader.cu:722-754)."""
    expected = expected_tensors(cfg)
    actual = {t.name: t for t in tensors}
    rep = InventoryReport()
    for name, shape in expected:
        t = actual.get(name)
        if t is None:
            rep.missing.append(name)
        elif t.shape != shape:
            rep.shape_mismatches.append(
                f"{name}: expected [{', '.join(map(str, shape))}] "
                f"got [{', '.join(map(str, t.shape))}]")
    names = {n for n, _ in expected}
    rep.unexpected = [t.name for t in tensors if t.name not in names]
    for lst in (rep.missing, rep.unexpected, rep.shape_mismatches):
        lst.sort()
    return rep


def inspect_checkpoint(model_dir: str | os.PathLike):
    """-> (config, tensors, data offset); raises VlasrInputError unless the
    checkpoint has exactly the official inventory."""
    model_dir = Path(model_dir)
    cfg = parse_model_config(model_dir)
    tensors, data_offset = read_safetensors_header(model_dir / "model.safetensors")
    # the projector width is not in config.json: take it from linear_1, so the
    # check is linear_2's input == linear_1's output (internal consistency)
    for t in tensors:
        if t.name == "multi_modal_projector.linear_1.weight":
            cfg = replace(cfg, projector_mid=t.shape[0])
    rep = validate_inventory(tensors, cfg)
    if not rep.ok:
        raise VlasrInputError(
            "checkpoint inventory does not match the official GLM-ASR layout: "
            + json.dumps(rep.to_json()))
    return cfg, tensors, data_offset


def load_weights(model_dir: str | os.PathLike, device, dtype=None, prefixes=None):
    """Resident device tensors of a validated checkpoint, name -> tensor.

    `prefixes` (e.g. ("audio_tower.", "multi_modal_projector.")) limits the
    upload to the named parts.  Tensors are views into one device arena with
    256-byte aligned slots (what cuBLAS wants for vector loads), in BF16, or
    converted on the device when `dtype` is given."""
    import torch
    cfg, tensors, data_offset = inspect_checkpoint(model_dir)
    if prefixes is not None:
        tensors = [t for t in tensors if t.name.startswith(tuple(prefixes))]
    slots, cursor = [], 0
    for t in tensors:
        slots.append(cursor)
        cursor += (t.nbytes + ARENA_ALIGN - 1) // ARENA_ALIGN * ARENA_ALIGN
    dev = torch.device(device)
    raw = torch.empty(cursor + ARENA_ALIGN, dtype=torch.uint8, device=dev)
    arena = raw[(-raw.data_ptr()) % ARENA_ALIGN:]          # 256-byte aligned base
    lo = min((t.begin for t in tensors), default=0)
    hi = max((t.end for t in tensors), default=0)
    mm = np.memmap(Path(model_dir) / "model.safetensors", dtype=np.uint8, mode="r",
                   offset=data_offset + lo, shape=(hi - lo,))
    pinned = torch.empty(hi - lo, dtype=torch.uint8, pin_memory=dev.type == "cuda")
    pinned.numpy()[:] = mm
    del mm
    out = {}
    for t, slot in zip(tensors, slots):
        dst = arena[slot:slot + t.nbytes]
        dst.copy_(pinned[t.begin - lo:t.end - lo], non_blocking=True)
        w = dst.view(torch.bfloat16).view(t.shape)
        out[t.name] = w if dtype is None or dtype == torch.bfloat16 else w.to(dtype)
    if dev.type == "cuda":
        torch.cuda.current_stream(dev).synchronize()
    return cfg, out


def write_checkpoint(model_dir: str | os.PathLike, cfg: AsrModelConfig, tensors: dict) -> None:
    """Write config.json + model.safetensors (BF16) from name -> array of
    uint16 BF16 bit patterns (numpy) with the given shapes."""
    model_dir = Path(model_dir)
    model_dir.mkdir(parents=True, exist_ok=True)
    (model_dir / "config.json").write_text(json.dumps(cfg.to_json(), indent=1))
    header, offset = {}, 0
    names = sorted(tensors)
    for name in names:
        a = tensors[name]
        if a.dtype != np.uint16:
            raise VlasrInputError(f"{name}: expected BF16 bit patterns (uint16)")
        header[name] = {"dtype": "BF16", "shape": list(a.shape),
                        "data_offsets": [offset, offset + a.nbytes]}
        offset += a.nbytes
    raw = json.dumps(header, separators=(",", ":")).encode()
    raw += b" " * (-len(raw) % 8)
    with open(model_dir / "model.safetensors", "wb") as f:
        f.write(len(raw).to_bytes(8, "little"))
        f.write(raw)
        for name in names:
            f.write(np.ascontiguousarray(tensors[name]).tobytes())
