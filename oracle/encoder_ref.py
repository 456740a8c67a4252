"""fp32 restatement of the reference's GLM-ASR audio tower + projector - TEST
INFRASTRUCTURE ONLY (the checker of vlasr.encoder; never on the product path).

Follows the batched encoder of VideoLingo-user native/asr/src/engine.cu,
run_encode_batched (:1166-1616), stage by stage, in float32 on the CPU with
no intermediate rounding:

* conv frontend (:1310-1330): im2col rows `x[cin][t-1+k]` (zero outside
  [0, T)) times the [hidden, cin*3] kernel, + bias, GELU; conv2 the same on
  `x[2t-1+k]` - exactly conv1d(padding 1) then conv1d(stride 2, padding 1);
* per layer (:1340-1580): LayerNorm (mean, E[x^2] - mean^2, eps 1e-5,
  :162-192), q/k/v projections (no k bias), partial RoPE on the first 32 of
  64 dims with pairs (d, d+16), cos/sin tables from fp64 angles cast to f32
  (:892-905) at position row % 1500 (:214-233), softmax(q k^T / 8) v per
  chunk and head (:1399-1412), o projection, residual add, post-attention
  LayerNorm, fc1 + bias, exact-erf GELU (:110-112), fc2 + bias, residual add;
* final LayerNorm, then the projector on 4 merged frames per token:
  linear_1 + bias, GELU, linear_2 + bias (:1583-1598).

The restatement is pinned against transformers' GlmAsrEncoder and
GlmAsrMultiModalProjector (the model the reference implements) by
tests/test_encoder_cpu.py.
"""

from __future__ import annotations

import math

import torch

MERGE = 4


def _ln(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    mean = x.mean(-1, keepdim=True)
    var = (x * x).mean(-1, keepdim=True) - mean * mean
    return (x - mean) * torch.rsqrt(var + eps) * w + b


def _gelu(x: torch.Tensor) -> torch.Tensor:
    return 0.5 * x * (1.0 + torch.erf(x * (1.0 / math.sqrt(2.0))))


def rope_tables(frames: int, rotary_dim: int, base: float = 10000.0):
    """cos/sin [frames, rotary_dim] from fp64 angles, cast to f32 (engine.cu:892-905)."""
    half = rotary_dim // 2
    d = torch.arange(rotary_dim, dtype=torch.float64) % half
    inv = 1.0 / torch.pow(torch.tensor(base, dtype=torch.float64), (2.0 * d) / rotary_dim)
    ang = torch.arange(frames, dtype=torch.float64)[:, None] * inv[None, :]
    return torch.cos(ang).float(), torch.sin(ang).float()


def _rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, rotary_dim: int) -> torch.Tensor:
    """x [C, frames, heads, head_dim]; rotate-half on the first rotary_dim dims."""
    half = rotary_dim // 2
    x = x.clone()
    x1 = x[..., :half].clone()
    x2 = x[..., half:rotary_dim].clone()
    c1, s1 = cos[None, :, None, :half], sin[None, :, None, :half]
    c2, s2 = cos[None, :, None, half:], sin[None, :, None, half:]
    x[..., :half] = x1 * c1 - x2 * s1
    x[..., half:rotary_dim] = x2 * c2 + x1 * s2
    return x


def encode_fp32(mel, weights: dict, heads: int = 20, layers: int | None = None,
                stages: bool = False, threads: int | None = None):
    """mel [C, bins, T] -> projector [C*T/8, out] (float32, CPU).

    `weights`: official tensor names -> tensors of any float dtype (cast to
    f32).  `layers` keeps the first layers only.  With stages=True returns
    {'conv_hidden', 'final_norm', 'projector'} like the reference's stage dumps.
    """
    if threads:
        torch.set_num_threads(threads)
    with torch.no_grad():
        W = {k: v.detach().to("cpu", torch.float32) for k, v in weights.items()
             if k.startswith(("audio_tower.", "multi_modal_projector."))}
        x = torch.as_tensor(mel).to("cpu", torch.float32)
        chunks = x.shape[0]
        hidden = W["audio_tower.conv1.weight"].shape[0]
        head_dim = hidden // heads
        rot = head_dim // 2
        n_layers = 0
        while f"audio_tower.layers.{n_layers}.mlp.fc1.weight" in W:
            n_layers += 1
        if layers is not None:
            n_layers = min(n_layers, layers)
        F = torch.nn.functional
        c1 = _gelu(F.conv1d(x, W["audio_tower.conv1.weight"], W["audio_tower.conv1.bias"],
                            padding=1))
        c2 = _gelu(F.conv1d(c1, W["audio_tower.conv2.weight"], W["audio_tower.conv2.bias"],
                            stride=2, padding=1))
        frames = c2.shape[-1]
        h = c2.transpose(1, 2).reshape(chunks * frames, hidden).contiguous()
        out = {"conv_hidden": h.clone()} if stages else {}
        cos, sin = rope_tables(frames, rot)
        scale = 1.0 / math.sqrt(head_dim)
        for l in range(n_layers):
            p = f"audio_tower.layers.{l}."
            y = _ln(h, W[p + "input_layernorm.weight"], W[p + "input_layernorm.bias"])
            q = y @ W[p + "self_attn.q_proj.weight"].T + W[p + "self_attn.q_proj.bias"]
            k = y @ W[p + "self_attn.k_proj.weight"].T
            v = y @ W[p + "self_attn.v_proj.weight"].T + W[p + "self_attn.v_proj.bias"]
            q = _rope(q.view(chunks, frames, heads, head_dim), cos, sin, rot)
            k = _rope(k.view(chunks, frames, heads, head_dim), cos, sin, rot)
            v = v.view(chunks, frames, heads, head_dim)
            q, k, v = (t.permute(0, 2, 1, 3) for t in (q, k, v))     # [C, heads, frames, hd]
            s = torch.matmul(q, k.transpose(-1, -2)) * scale
            pr = torch.softmax(s, dim=-1)
            a = torch.matmul(pr, v).permute(0, 2, 1, 3).reshape(chunks * frames, hidden)
            h = h + (a @ W[p + "self_attn.o_proj.weight"].T + W[p + "self_attn.o_proj.bias"])
            y = _ln(h, W[p + "post_attention_layernorm.weight"],
                    W[p + "post_attention_layernorm.bias"])
            f = _gelu(y @ W[p + "mlp.fc1.weight"].T + W[p + "mlp.fc1.bias"])
            h = h + (f @ W[p + "mlp.fc2.weight"].T + W[p + "mlp.fc2.bias"])
        z = _ln(h, W["audio_tower.norm.weight"], W["audio_tower.norm.bias"])
        if stages:
            out["final_norm"] = z.clone()
        zt = z.view(chunks * frames // MERGE, MERGE * hidden)
        pm = _gelu(zt @ W["multi_modal_projector.linear_1.weight"].T
                   + W["multi_modal_projector.linear_1.bias"])
        proj = (pm @ W["multi_modal_projector.linear_2.weight"].T
                + W["multi_modal_projector.linear_2.bias"])
        if stages:
            out["projector"] = proj
            return out
        return proj
