"""GLM-ASR audio tower + projector on one GPU: the encoder-layer caller of the
fused layer ops.

A host loop over resident weights that computes what the reference's batched
encoder computes (VideoLingo-user native/asr/src/engine.cu:1166-1616,
run_encode_batched; the same model as transformers' GlmAsrEncoder and
GlmAsrMultiModalProjector):

    mel [C,128,3000] -> conv1(k3,s1,p1) + GELU -> conv2(k3,s2,p1) + GELU -> h [C*1500,1280]
    32 x {  y     = LN1(h)                 fused with the previous layer's residual add
            qkv   = y Wqkv^T + b           one GEMM (k has no bias)
            RoPE(q, k) in place            rotary 32 of 64 dims, position = frame
            a     = softmax(q k^T / 8) v   unmasked, per chunk and head
            h    += a Wo^T + bo;  y = LN2(h)          one fused add+LN launch
            f     = GELU(y W1^T + b1)      bias fused into the GELU launch
            delta = f W2^T + b2 }          added into h by the next LN launch
    z = LN(h + delta) -> [C*375, 5120] -> GELU(z W^T + b) -> (.) W^T + b -> [C*375, 2048]

The memory-bound steps are this library's kernels (add+LayerNorm, GELU with
bias, RoPE): 65 + 35 + 32 launches per pass.  GEMMs go to cuBLAS and the conv
frontend to cuDNN (NHWC, so conv2's output already is the [frames, hidden]
row layout), attention to torch's fused SDPA.  Compared with the reference:
every GEMM accumulates in fp32 (the reference defaults to fp16 accumulation;
its `--gemm-acc 32` mode matches), attention keeps scores and probabilities
on chip in fp32 (the reference materialises them in fp16), and q/k/v come
from one GEMM instead of three.
"""

from __future__ import annotations

import contextlib
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import ops
from ._lib import VlasrInputError

MERGE = 4          # encoder frames merged per projector token


@dataclass(frozen=True)
class EncoderShape:
    mel_bins: int
    hidden: int
    heads: int
    head_dim: int
    ffn: int
    layers: int
    proj_mid: int
    out_dim: int
    rotary_dim: int
    rope_base: float = 10000.0
    eps: float = 1e-5


def _shape_from(weights: dict, heads: int) -> EncoderShape:
    w1 = weights["audio_tower.conv1.weight"]
    hidden, mel_bins = w1.shape[0], w1.shape[1]
    layers = 0
    while f"audio_tower.layers.{layers}.mlp.fc1.weight" in weights:
        layers += 1
    if hidden % heads:
        raise VlasrInputError("hidden size must be a multiple of the head count")
    head_dim = hidden // heads
    return EncoderShape(
        mel_bins=mel_bins, hidden=hidden, heads=heads, head_dim=head_dim,
        ffn=weights["audio_tower.layers.0.mlp.fc1.weight"].shape[0] if layers else 0,
        layers=layers,
        proj_mid=weights["multi_modal_projector.linear_1.weight"].shape[0],
        out_dim=weights["multi_modal_projector.linear_2.weight"].shape[0],
        rotary_dim=head_dim // 2)       # partial_rotary_factor 0.5


def flops_per_chunk(s: EncoderShape, mel_frames: int = 3000) -> int:
    """Multiply-add FLOPs (2 per MAC) of one chunk: conv frontend, per layer
    the q/k/v/o and MLP GEMMs plus q k^T and p v, and the projector."""
    frames = (mel_frames - 1) // 2 + 1
    conv = 2 * mel_frames * s.hidden * s.mel_bins * 3 + 2 * frames * s.hidden * s.hidden * 3
    layer = (2 * frames * (4 * s.hidden * s.hidden + 2 * s.hidden * s.ffn)
             + 2 * 2 * s.heads * frames * frames * s.head_dim)
    proj = 2 * (frames // MERGE) * (MERGE * s.hidden * s.proj_mid + s.proj_mid * s.out_dim)
    return conv + s.layers * layer + proj


_SDPA = {"flash": "FLASH_ATTENTION", "cudnn": "CUDNN_ATTENTION",
         "efficient": "EFFICIENT_ATTENTION", "math": "MATH"}


class AudioEncoder:
    """Resident weights in one compute dtype (bf16 or fp16) and the launch
    sequence of the audio tower + projector.

    `weights` maps the official tensor names (audio_tower.*,
    multi_modal_projector.*) to device tensors, e.g. from
    vlasr.checkpoint.load_weights; `layers` keeps only the first layers
    (tests).  Buffers are allocated per chunk count and reused."""

    def __init__(self, weights: dict, *, heads: int = 20, dtype=torch.bfloat16,
                 layers: int | None = None, attention: str = "auto"):
        if dtype not in (torch.bfloat16, torch.float16):
            raise VlasrInputError("AudioEncoder computes in bf16 or fp16")
        if attention != "auto" and attention not in _SDPA:
            raise VlasrInputError(f"attention must be 'auto' or one of {sorted(_SDPA)}")
        self.dtype = dtype
        self.attention = attention
        s = _shape_from(weights, heads)
        if layers is not None:
            if not 0 <= layers <= s.layers:
                raise VlasrInputError(f"layers must be in [0, {s.layers}]")
            s = EncoderShape(**{**s.__dict__, "layers": layers})
        if s.proj_mid and weights["multi_modal_projector.linear_1.weight"].shape[1] != MERGE * s.hidden:
            raise VlasrInputError("projector linear_1 must take 4 merged frames")
        self.shape = s
        dev = weights["audio_tower.conv1.weight"].device
        if dev.type != "cuda":
            raise VlasrInputError("AudioEncoder weights must be CUDA tensors")
        self.device = dev

        def w(name):
            return weights[name].to(device=dev, dtype=dtype).contiguous()

        cl = torch.channels_last
        # conv kernels as [out, in, 1, 3] NHWC filters
        self.conv1_w = w("audio_tower.conv1.weight").unsqueeze(2).contiguous(memory_format=cl)
        self.conv1_b = w("audio_tower.conv1.bias")
        self.conv2_w = w("audio_tower.conv2.weight").unsqueeze(2).contiguous(memory_format=cl)
        self.conv2_b = w("audio_tower.conv2.bias")
        self.layer_w = []
        for l in range(s.layers):
            p = f"audio_tower.layers.{l}."
            wq, wk, wv = (w(p + f"self_attn.{n}_proj.weight") for n in "qkv")
            bq, bv = w(p + "self_attn.q_proj.bias"), w(p + "self_attn.v_proj.bias")
            self.layer_w.append({
                "ln1_w": w(p + "input_layernorm.weight"), "ln1_b": w(p + "input_layernorm.bias"),
                "qkv_wt": torch.cat([wq, wk, wv], 0).t(),          # [hidden, 3*hidden] view
                "qkv_b": torch.cat([bq, torch.zeros_like(bq), bv]),
                "o_wt": w(p + "self_attn.o_proj.weight").t(), "o_b": w(p + "self_attn.o_proj.bias"),
                "ln2_w": w(p + "post_attention_layernorm.weight"),
                "ln2_b": w(p + "post_attention_layernorm.bias"),
                "fc1_wt": w(p + "mlp.fc1.weight").t(), "fc1_b": w(p + "mlp.fc1.bias"),
                "fc2_wt": w(p + "mlp.fc2.weight").t(), "fc2_b": w(p + "mlp.fc2.bias"),
            })
        self.norm_w, self.norm_b = w("audio_tower.norm.weight"), w("audio_tower.norm.bias")
        self.p1_wt = w("multi_modal_projector.linear_1.weight").t()
        self.p1_b = w("multi_modal_projector.linear_1.bias")
        self.p2_wt = w("multi_modal_projector.linear_2.weight").t()
        self.p2_b = w("multi_modal_projector.linear_2.bias")
        self._bufs: dict = {}

    # ------------------------------------------------------------------
    def _buffers(self, chunks: int, mel_frames: int) -> dict:
        key = (chunks, mel_frames)
        if key not in self._bufs:
            s, dt, dev = self.shape, self.dtype, self.device
            frames = (mel_frames - 1) // 2 + 1
            rows = chunks * frames
            self._bufs = {key: {
                "frames": frames,
                "h": torch.empty(rows, s.hidden, dtype=dt, device=dev),
                "y": torch.empty(rows, s.hidden, dtype=dt, device=dev),
                "qkv": torch.empty(rows, 3 * s.hidden, dtype=dt, device=dev),
                "o": torch.empty(rows, s.hidden, dtype=dt, device=dev),
                "f": torch.empty(rows, s.ffn, dtype=dt, device=dev),
                "p": torch.empty(rows // MERGE, s.proj_mid, dtype=dt, device=dev),
            }}
        return self._bufs[key]

    def conv_frontend(self, mel: torch.Tensor, h: torch.Tensor) -> None:
        """mel [C, bins, T] -> GELU(conv2(GELU(conv1(mel)))) as rows [C*T', hidden] in h."""
        c, bins, t = mel.shape
        x = mel.to(self.dtype).unsqueeze(2).contiguous(memory_format=torch.channels_last)
        cl = torch.channels_last
        c1 = F.conv2d(x, self.conv1_w, self.conv1_b, padding=(0, 1)).contiguous(memory_format=cl)
        c1v = c1.permute(0, 2, 3, 1)                     # [C, 1, T, hidden], row-major
        ops.gelu_erf(c1v, out=c1v)
        c2 = F.conv2d(c1, self.conv2_w, self.conv2_b, stride=(1, 2), padding=(0, 1))
        c2v = c2.contiguous(memory_format=cl).permute(0, 2, 3, 1).reshape(h.shape)
        ops.gelu_erf(c2v, out=h)

    def encode(self, mel: torch.Tensor, stages: bool = False):
        """mel [C, 128, 3000] (f32 or the compute dtype, on the device) ->
        projector output [C*375, 2048] in the compute dtype.

        With stages=True returns a dict with the conv frontend output
        ('conv_hidden'), the final LayerNorm ('final_norm') and the projector
        ('projector'), like the reference's EncodeOutput stage dumps."""
        s = self.shape
        if mel.dim() != 3 or mel.shape[1] != s.mel_bins or not mel.is_cuda:
            raise VlasrInputError(f"mel must be a CUDA tensor [chunks, {s.mel_bins}, frames]")
        chunks, _, mel_frames = mel.shape
        b = self._buffers(chunks, mel_frames)
        frames = b["frames"]
        if frames % MERGE:
            raise VlasrInputError("frames per chunk must merge into whole projector tokens")
        h, y, qkv, o, f = b["h"], b["y"], b["qkv"], b["o"], b["f"]
        hs, nh, hd = s.hidden, s.heads, s.head_dim
        out = {}
        if self.attention == "auto":
            sdpa_ctx = contextlib.nullcontext
        else:
            from torch.nn.attention import SDPBackend, sdpa_kernel
            backend = getattr(SDPBackend, _SDPA[self.attention])
            sdpa_ctx = lambda: sdpa_kernel([backend])  # noqa: E731
        self.conv_frontend(mel, h)
        if stages:
            out["conv_hidden"] = h.clone()
        delta = None
        for lw in self.layer_w:
            ops.add_layernorm(h, delta, lw["ln1_w"], lw["ln1_b"], eps=s.eps, out=y)
            torch.addmm(lw["qkv_b"], y, lw["qkv_wt"], out=qkv)
            ops.rope_(qkv[:, :hs], qkv[:, hs:2 * hs], head_dim=hd, rotary_dim=s.rotary_dim,
                      base=s.rope_base, seq_len=frames)
            q, k, v = (qkv[:, i * hs:(i + 1) * hs].view(chunks, frames, nh, hd).transpose(1, 2)
                       for i in range(3))
            with sdpa_ctx():
                a = F.scaled_dot_product_attention(q, k, v)       # [C, heads, frames, hd]
            a = a.transpose(1, 2).reshape(chunks * frames, hs)
            torch.addmm(lw["o_b"], a, lw["o_wt"], out=o)
            ops.add_layernorm(h, o, lw["ln2_w"], lw["ln2_b"], eps=s.eps, out=y)
            torch.mm(y, lw["fc1_wt"], out=f)
            ops.gelu_erf(f, lw["fc1_b"], out=f)
            torch.addmm(lw["fc2_b"], f, lw["fc2_wt"], out=o)
            delta = o
        z = ops.add_layernorm(h, delta, self.norm_w, self.norm_b, eps=s.eps, out=y)
        if stages:
            out["final_norm"] = z.clone()
        zt = z.view(chunks * frames // MERGE, MERGE * hs)
        p = torch.mm(zt, self.p1_wt, out=b["p"])
        ops.gelu_erf(p, self.p1_b, out=p)
        proj = torch.addmm(self.p2_b, p, self.p2_wt)
        if stages:
            out["projector"] = proj
            return out
        return proj

    def launches_per_pass(self) -> int:
        """Kernels of this library one encode() launches."""
        return 2 + self.shape.layers * 4 + 2
