"""Tensor-level API over libvlasr.so.

PyTorch tensors are only buffer carriers here: every op hands raw device
pointers, shapes and the current CUDA stream to the C ABI and returns the
output tensor.  Nothing falls back to a PyTorch or CPU implementation; a
CPU tensor or a missing library is an error.

Op semantics and their reference kernels (VideoLingo-user native/asr/src):

=====================  ==========================================================
add_layernorm          residual_add_kernel + layer_norm_kernel (engine.cu:162-212)
add_rmsnorm            residual_add_kernel + rmsnorm_kernel (decoder.cu:81-101,933-938)
gelu_erf               add_bias_kernel + gelu_kernel (engine.cu:110-112,194-205)
swiglu                 silu_mul_kernel (decoder.cu:103-109)
rope_                  rope_kernel, rope_rows/rope_full/rope_at_position* kernels
                       (engine.cu:214-233; decoder.cu:113-134,307-333,471-498,670-695,789-814)
embed_gather           gather_inputs/gather_batch/gather_ids_* kernels
                       (decoder.cu:60-78,460-469,636-667)
kv_append              append_kv* kernels (decoder.cu:335-351,500-514,857-882,940-948)
rope_kv_append         rope_at_position_map_kernel + append_kv_mapped_kernel fused
logmel                 compute_mel_batched (mel_frontend.cu:209-291)
=====================  ==========================================================
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import VL_BF16, VL_F16, VL_F32, VlasrInputError, check

MEL_BINS = 128
MEL_FRAMES = 3000
CHUNK_SAMPLES = 480000

_DTYPES = {torch.float32: VL_F32, torch.float16: VL_F16, torch.bfloat16: VL_BF16}


def _dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise VlasrInputError(f"unsupported dtype {t.dtype}; expected float32/float16/bfloat16")


def _cuda(t: torch.Tensor, name: str) -> torch.Tensor:
    if not isinstance(t, torch.Tensor):
        raise VlasrInputError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise VlasrInputError(f"{name} must be a CUDA tensor (there is no CPU path)")
    return t


def _contig(t: torch.Tensor, name: str) -> torch.Tensor:
    _cuda(t, name)
    if not t.is_contiguous():
        raise VlasrInputError(f"{name} must be contiguous")
    return t


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _same(ref: torch.Tensor, t: torch.Tensor | None, name: str) -> None:
    if t is None:
        return
    if t.dtype != ref.dtype or t.device != ref.device:
        raise VlasrInputError(f"{name} must match dtype/device {ref.dtype}/{ref.device}")


# ---------------------------------------------------------------------------
# Norms
# ---------------------------------------------------------------------------

def init(device: torch.device | int | None = None) -> None:
    """Once-per-device set-up (vl_init): builds the GELU tables and the
    kernels' attributes ahead of the first op call, e.g. before capturing a
    CUDA graph.  Optional - every op does its own part on first use."""
    if device is None:
        idx = torch.cuda.current_device()
    elif isinstance(device, int):
        idx = device
    else:
        idx = torch.device(device).index
        idx = torch.cuda.current_device() if idx is None else idx
    check(_lib.load().vl_init(int(idx)), "vl_init")


def add_layernorm(residual: torch.Tensor, delta: torch.Tensor | None, gamma: torch.Tensor,
                  beta: torch.Tensor | None, eps: float = 1e-5,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """h = round(residual + delta) (written back into residual); out = LayerNorm(h).

    With delta None, out = LayerNorm(residual) and residual is not modified
    (pass out=residual for the reference's in-place layer_norm_kernel).
    """
    _contig(residual, "residual")
    cols = residual.shape[-1]
    rows = residual.numel() // cols if cols else 0
    for name, t in (("delta", delta), ("gamma", gamma), ("beta", beta)):
        if t is not None:
            _contig(t, name)
            _same(residual, t, name)
    if gamma.numel() != cols or (beta is not None and beta.numel() != cols):
        raise VlasrInputError("gamma/beta must have residual.shape[-1] elements")
    if delta is not None and delta.shape != residual.shape:
        raise VlasrInputError("delta must have the residual's shape")
    if out is None:
        out = torch.empty_like(residual)
    _contig(out, "out")
    _same(residual, out, "out")
    if out.shape != residual.shape:
        raise VlasrInputError("out must have the residual's shape")
    check(_lib.load().vl_add_layernorm(_ptr(residual), _ptr(delta), _ptr(gamma), _ptr(beta),
                                       _ptr(out), rows, cols, float(eps), _dtype_code(residual),
                                       _stream(residual)), "vl_add_layernorm")
    return out


def add_rmsnorm(residual: torch.Tensor, delta: torch.Tensor | None, weight: torch.Tensor,
                eps: float = 1e-5, out: torch.Tensor | None = None) -> torch.Tensor:
    """h = round(residual + delta) (written back into residual); out = RMSNorm(h)."""
    _contig(residual, "residual")
    cols = residual.shape[-1]
    rows = residual.numel() // cols if cols else 0
    for name, t in (("delta", delta), ("weight", weight)):
        if t is not None:
            _contig(t, name)
            _same(residual, t, name)
    if weight.numel() != cols:
        raise VlasrInputError("weight must have residual.shape[-1] elements")
    if delta is not None and delta.shape != residual.shape:
        raise VlasrInputError("delta must have the residual's shape")
    if out is None:
        out = torch.empty_like(residual)
    _contig(out, "out")
    _same(residual, out, "out")
    if out.shape != residual.shape:
        raise VlasrInputError("out must have the residual's shape")
    check(_lib.load().vl_add_rmsnorm(_ptr(residual), _ptr(delta), _ptr(weight), _ptr(out), rows,
                                     cols, float(eps), _dtype_code(residual), _stream(residual)),
          "vl_add_rmsnorm")
    return out


# ---------------------------------------------------------------------------
# Activations
# ---------------------------------------------------------------------------

def gelu_erf(x: torch.Tensor, bias: torch.Tensor | None = None,
             out: torch.Tensor | None = None) -> torch.Tensor:
    """Exact-erf GELU of x (+ bias over the last dim, rounded before GELU)."""
    _contig(x, "x")
    cols = x.shape[-1] if x.dim() else 1
    rows = x.numel() // cols if cols else 0
    if bias is not None:
        _contig(bias, "bias")
        _same(x, bias, "bias")
        if bias.numel() != cols:
            raise VlasrInputError("bias must have x.shape[-1] elements")
    if out is None:
        out = torch.empty_like(x)
    _contig(out, "out")
    _same(x, out, "out")
    if out.shape != x.shape:
        raise VlasrInputError("out must have x's shape")
    check(_lib.load().vl_gelu_erf(_ptr(x), _ptr(bias), _ptr(out), rows, cols, _dtype_code(x),
                                  _stream(x)), "vl_gelu_erf")
    return out


def _rows2d(t: torch.Tensor, name: str, cols: int) -> torch.Tensor:
    """View t as [rows, cols] with contiguous rows (a row stride is allowed)."""
    if t.is_contiguous():
        return t.reshape(-1, cols)
    if t.dim() == 2 and t.stride(1) == 1:
        return t
    raise VlasrInputError(f"{name} must be contiguous or a 2-D view with contiguous rows")


def swiglu(gate: torch.Tensor, up: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """out = silu(gate) * up.  gate/up may be row-strided 2-D views (e.g. the
    halves of a packed [rows, 2*cols] buffer); out=gate reproduces the
    reference's in-place silu_mul_kernel."""
    _cuda(gate, "gate")
    _cuda(up, "up")
    _same(gate, up, "up")
    if gate.shape != up.shape or gate.dim() < 1:
        raise VlasrInputError("gate and up must have the same shape")
    cols = gate.shape[-1]
    g2, u2 = _rows2d(gate, "gate", cols), _rows2d(up, "up", cols)
    if out is None:
        out = torch.empty(gate.shape, dtype=gate.dtype, device=gate.device)
    _cuda(out, "out")
    _same(gate, out, "out")
    o2 = _rows2d(out, "out", cols)
    if o2.shape != g2.shape:
        raise VlasrInputError("out must have gate's shape")
    check(_lib.load().vl_swiglu(_ptr(g2), _ptr(u2), _ptr(o2), g2.shape[0], cols, g2.stride(0),
                                u2.stride(0), o2.stride(0), _dtype_code(gate), _stream(gate)),
          "vl_swiglu")
    return out


# ---------------------------------------------------------------------------
# RoPE
# ---------------------------------------------------------------------------

def _heads_view(t: torch.Tensor, head_dim: int, name: str):
    """[tokens, heads, head_dim] (or [..., heads*head_dim]) -> (tokens, heads, row_stride)."""
    _cuda(t, name)
    if t.stride(-1) != 1:
        raise VlasrInputError(f"{name} must have a contiguous last dim")
    if t.dim() >= 3 and t.shape[-1] == head_dim:
        heads = t.shape[-2]
        if t.stride(-2) != head_dim:
            raise VlasrInputError(f"{name} heads must be packed")
        lead = t.shape[:-2]
        row_stride = t.stride(-3)
    else:
        if t.shape[-1] % head_dim:
            raise VlasrInputError(f"{name}.shape[-1] must be a multiple of head_dim")
        heads = t.shape[-1] // head_dim
        lead = t.shape[:-1]
        row_stride = t.stride(-2) if t.dim() >= 2 else t.shape[-1]
    tokens = 1
    for s in lead:
        tokens *= s
    if len(lead) > 1:
        # leading dims must collapse into one uniform row stride
        exp = row_stride
        for d in range(len(lead) - 1, 0, -1):
            exp *= lead[d]
            if t.stride(d - 1) != exp:
                raise VlasrInputError(f"{name} leading dims must be row-uniform")
    return tokens, heads, row_stride


def rope_(q: torch.Tensor, k: torch.Tensor | None, *, head_dim: int, rotary_dim: int | None = None,
          base: float = 10000.0, positions: torch.Tensor | None = None,
          row_map: torch.Tensor | None = None, positions_stride: int = 1, pos_offset: int = 0,
          seq_len: int = 0) -> None:
    """Rotate-half RoPE on q (and k) in place.

    Row r uses pos_offset + positions[row_map[r] * positions_stride] when
    positions is given, else pos_offset + (r % seq_len if seq_len else r).
    """
    rotary_dim = head_dim if rotary_dim is None else rotary_dim
    tokens, nq, qs = _heads_view(q, head_dim, "q")
    nk, ks = 0, 0
    if k is not None:
        _same(q, k, "k")
        kt, nk, ks = _heads_view(k, head_dim, "k")
        if kt != tokens:
            raise VlasrInputError("q and k must have the same number of tokens")
    for name, t in (("positions", positions), ("row_map", row_map)):
        if t is not None:
            _contig(t, name)
            if t.dtype != torch.int32:
                raise VlasrInputError(f"{name} must be int32")
    check(_lib.load().vl_rope_inplace(_ptr(q), _ptr(k), _ptr(positions), _ptr(row_map),
                                      positions_stride, pos_offset, tokens, seq_len, nq, nk,
                                      head_dim, rotary_dim, float(base), qs, ks, _dtype_code(q),
                                      _stream(q)), "vl_rope_inplace")


def rope_kv_append(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, k_cache: torch.Tensor,
                   v_cache: torch.Tensor, positions: torch.Tensor, slot_mapping: torch.Tensor, *,
                   head_dim: int, rotary_dim: int | None = None, base: float = 10000.0,
                   status: torch.Tensor | None = None) -> None:
    """Decode step: rotate q, k in place at `positions`, store k and v at `slot_mapping`."""
    rotary_dim = head_dim if rotary_dim is None else rotary_dim
    for name, t in (("q", q), ("k", k), ("v", v), ("k_cache", k_cache), ("v_cache", v_cache)):
        _contig(t, name)
        _same(q, t, name)
    tokens = positions.numel()
    nq = q.numel() // (tokens * head_dim) if tokens else 0
    nk = k.numel() // (tokens * head_dim) if tokens else 0
    if v.numel() != k.numel() or k_cache.shape != v_cache.shape:
        raise VlasrInputError("k/v and k_cache/v_cache must match")
    num_slots = k_cache.numel() // (nk * head_dim) if nk else 0
    _contig(positions, "positions")
    _contig(slot_mapping, "slot_mapping")
    if positions.dtype != torch.int32 or slot_mapping.dtype != torch.int64:
        raise VlasrInputError("positions must be int32 and slot_mapping int64")
    if slot_mapping.numel() != tokens:
        raise VlasrInputError("slot_mapping must have one entry per token")
    check(_lib.load().vl_rope_kv_append(_ptr(q), _ptr(k), _ptr(v), _ptr(k_cache), _ptr(v_cache),
                                        _ptr(positions), _ptr(slot_mapping), tokens, nq, nk,
                                        head_dim, rotary_dim, float(base), num_slots,
                                        _dtype_code(q), _ptr(status), _stream(q)),
          "vl_rope_kv_append")


def decode_rows(residual: torch.Tensor, delta: torch.Tensor | None, weight: torch.Tensor,
                q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, k_cache: torch.Tensor,
                v_cache: torch.Tensor, positions: torch.Tensor, slot_mapping: torch.Tensor, *,
                head_dim: int, rotary_dim: int | None = None, base: float = 10000.0,
                eps: float = 1e-5, out: torch.Tensor | None = None,
                status: torch.Tensor | None = None) -> torch.Tensor:
    """The row ops of a decode step in one launch (vl_decode_rows): residual
    add + RMSNorm of `residual` [rows, cols] (as add_rmsnorm) and, side by
    side, RoPE of q/k at `positions` with the KV append at `slot_mapping`
    (as rope_kv_append).  q [tokens, n_q*head_dim], k/v [tokens,
    n_kv*head_dim] (contiguous rows), caches [num_slots, n_kv, head_dim].
    Returns the normalised rows."""
    rotary_dim = head_dim if rotary_dim is None else rotary_dim
    _contig(residual, "residual")
    if residual.dim() != 2:
        raise VlasrInputError("residual must be [rows, cols]")
    rows, cols = residual.shape
    for name, t in (("delta", delta), ("weight", weight), ("q", q), ("k", k), ("v", v),
                    ("k_cache", k_cache), ("v_cache", v_cache)):
        if t is not None:
            _contig(t, name)
            _same(residual, t, name)
    if out is None:
        out = torch.empty_like(residual)
    _contig(out, "out")
    _same(residual, out, "out")
    tokens = positions.numel()
    if q.dim() != 2 or k.dim() != 2 or v.shape != k.shape or q.shape[0] != tokens:
        raise VlasrInputError("q must be [tokens, n_q*head_dim], k and v [tokens, n_kv*head_dim]")
    if q.shape[1] % head_dim or k.shape[1] % head_dim:
        raise VlasrInputError("q/k widths must be multiples of head_dim")
    nq, nk = q.shape[1] // head_dim, k.shape[1] // head_dim
    if k_cache.shape != v_cache.shape or k_cache.numel() % (nk * head_dim):
        raise VlasrInputError("k_cache/v_cache must be [num_slots, n_kv, head_dim]")
    num_slots = k_cache.numel() // (nk * head_dim)
    _contig(positions, "positions")
    _contig(slot_mapping, "slot_mapping")
    if positions.dtype != torch.int32 or slot_mapping.dtype != torch.int64:
        raise VlasrInputError("positions must be int32 and slot_mapping int64")
    if slot_mapping.numel() != tokens:
        raise VlasrInputError("slot_mapping must have one entry per token")
    check(_lib.load().vl_decode_rows(
        _ptr(residual), _ptr(delta), _ptr(weight), _ptr(out), rows, cols, float(eps), _ptr(q),
        _ptr(k), _ptr(v), _ptr(k_cache), _ptr(v_cache), _ptr(positions), _ptr(slot_mapping),
        tokens, nq, nk, head_dim, rotary_dim, float(base), q.shape[1], k.shape[1], num_slots,
        _dtype_code(residual), _ptr(status), _stream(residual)), "vl_decode_rows")
    return out


# ---------------------------------------------------------------------------
# Decode-step attention
# ---------------------------------------------------------------------------

def decode_attention_workspace_bytes(tokens: int, n_q_heads: int, n_kv_heads: int,
                                     head_dim: int, max_seq_len: int) -> int:
    return int(_lib.load().vl_decode_attention_workspace_bytes(tokens, n_q_heads, n_kv_heads,
                                                               head_dim, max_seq_len))


_attn_ws: dict = {}


def _attn_workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """A zero-filled workspace per device, grown on demand (calls in stream
    order leave it zero-filled)."""
    key = (device.type, device.index)
    ws = _attn_ws.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=device)
        _attn_ws[key] = ws
    return ws


def _rows_of(t: torch.Tensor, width: int, name: str) -> tuple[int, int]:
    """(rows, row stride) of t viewed as rows of `width` contiguous elements."""
    _cuda(t, name)
    if t.stride(-1) != 1:
        raise VlasrInputError(f"{name} must have a contiguous last dim")
    if t.dim() >= 3:
        inner = t.shape[-1] * t.shape[-2]
        if inner != width or t.stride(-2) != t.shape[-1]:
            raise VlasrInputError(f"{name} rows must be [heads, head_dim] packed ({width} elements)")
        lead = t.shape[:-2]
        stride = t.stride(-3)
    else:
        if t.shape[-1] != width:
            raise VlasrInputError(f"{name} rows must have {width} elements")
        lead = t.shape[:-1]
        stride = t.stride(-2) if t.dim() == 2 else width
    rows = 1
    for d in lead:
        rows *= d
    if len(lead) > 1 and not t.is_contiguous():
        raise VlasrInputError(f"{name} leading dims must be contiguous")
    return rows, stride


def decode_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                     positions: torch.Tensor, seq_start: torch.Tensor, *, n_kv_heads: int,
                     head_dim: int, max_seq_len: int, k: torch.Tensor | None = None,
                     v: torch.Tensor | None = None, rotary_dim: int = 0,
                     rope_base: float = 10000.0, scale: float = 0.0,
                     out: torch.Tensor | None = None,
                     workspace: torch.Tensor | None = None,
                     status: torch.Tensor | None = None, pdl: bool = False) -> torch.Tensor:
    """One decode step of attention (vl_decode_attention).

    q [tokens, n_q_heads*head_dim] (or [tokens, n_q_heads, head_dim]; a row
    stride is allowed, e.g. a view of a packed qkv buffer); k_cache /
    v_cache [num_slots, n_kv_heads*head_dim] (or 3-D); positions int32
    [tokens]; seq_start int64 [tokens].  With k / v (new rows, same layout
    rules) RoPE at the positions (rotary_dim > 0) and the cache append are
    fused in.  max_seq_len bounds positions + 1 (a sequence's cache capacity):
    it sizes the split of the positions over CTAs, so pass the real bound.
    Without `workspace`, a zero-filled per-device workspace is used, which
    serves calls in stream order on one stream.  pdl=True launches it as a
    programmatic dependent of the previous kernel on the stream
    (VL_LAUNCH_PDL): that kernel must not write positions, seq_start or,
    with k / v, the cache rows before the positions."""
    _same(q, k_cache, "k_cache")
    _same(q, v_cache, "v_cache")
    kvw = n_kv_heads * head_dim
    num_slots, cs = _rows_of(k_cache, kvw, "k_cache")
    vslots, vs = _rows_of(v_cache, kvw, "v_cache")
    if (vslots, vs) != (num_slots, cs):
        raise VlasrInputError("k_cache and v_cache must have the same shape and row stride")
    qw = q.shape[-1] * (q.shape[-2] if q.dim() >= 3 else 1)
    if qw % head_dim:
        raise VlasrInputError("q rows must be a whole number of heads")
    nq = qw // head_dim
    tokens, qs = _rows_of(q, qw, "q")
    ks = 0
    if (k is None) != (v is None):
        raise VlasrInputError("k and v must both be given or both be None")
    if k is not None:
        _same(q, k, "k")
        _same(q, v, "v")
        kt, ks = _rows_of(k, kvw, "k")
        vt, vstr = _rows_of(v, kvw, "v")
        if kt != tokens or vt != tokens or vstr != ks:
            raise VlasrInputError("k and v must have one row per token and the same row stride")
    for name, t, dt in (("positions", positions, torch.int32), ("seq_start", seq_start, torch.int64)):
        _contig(t, name)
        if t.dtype != dt or t.numel() != tokens:
            raise VlasrInputError(f"{name} must be {dt} with one entry per token")
    max_seq_len = int(max_seq_len)
    if out is None:
        out = torch.empty((tokens, nq * head_dim), dtype=q.dtype, device=q.device)
    _same(q, out, "out")
    ot, os_ = _rows_of(out, nq * head_dim, "out")
    if ot != tokens:
        raise VlasrInputError("out must have one row per token")
    need = decode_attention_workspace_bytes(max(tokens, 1), nq, n_kv_heads, head_dim,
                                            max(max_seq_len, 1))
    if workspace is None:
        workspace = _attn_workspace(q.device, need)
    check(_lib.load().vl_decode_attention(
        _ptr(q), _ptr(k), _ptr(v), _ptr(k_cache), _ptr(v_cache), _ptr(positions),
        _ptr(seq_start), tokens, nq, n_kv_heads, head_dim, rotary_dim, float(rope_base),
        float(scale), qs, ks, cs, max_seq_len, num_slots, _ptr(out), os_, _dtype_code(q),
        _ptr(workspace), workspace.numel() * workspace.element_size(), _ptr(status),
        LAUNCH_PDL if pdl else 0, _stream(q)), "vl_decode_attention")
    return out


# ---------------------------------------------------------------------------
# Decode-step linear layers
# ---------------------------------------------------------------------------

LINEAR_EPILOGUES = {"store": 0, "swiglu": 1, "residual": 2}
LAUNCH_PDL = 1        # VL_LAUNCH_PDL
LINEAR_TCGEN05 = 2    # VL_LINEAR_TCGEN05
LINEAR_MAX_ROWS = 64


def decode_linear(x: torch.Tensor, w: torch.Tensor, *, epilogue: str = "store",
                  out: torch.Tensor | None = None, norm_weight: torch.Tensor | None = None,
                  ssq_in: torch.Tensor | None = None, eps: float = 1e-5,
                  ssq_out: torch.Tensor | None = None, pdl: bool = False,
                  tcgen05: bool = False) -> torch.Tensor:
    """y = x W^T for at most 64 token rows (vl_decode_linear).

    x [rows, k] (a row stride is allowed), w [n, k].  epilogue "store" -> out
    [rows, n]; "swiglu" (w = [gate; up]) -> out [rows, n/2]; "residual" ->
    out is the residual stream [rows, n], updated in place, and ssq_out
    (float32 [n/16, rows]) receives its per-16-column sums of squares.
    norm_weight + ssq_in (float32 [parts, rows], such partial sums) apply
    the RMSNorm prologue to x.  pdl=True launches it as a programmatic
    dependent of the previous kernel on the stream (VL_LAUNCH_PDL): that
    kernel must not write w or norm_weight.  tcgen05=True asks for the
    5th-generation tensor-core kernel (VL_LINEAR_TCGEN05; output columns in
    multiples of 128, otherwise ignored); the default kernel is faster."""
    if epilogue not in LINEAR_EPILOGUES:
        raise VlasrInputError(f"epilogue must be one of {sorted(LINEAR_EPILOGUES)}")
    _cuda(x, "x")
    _contig(w, "w")
    _same(x, w, "w")
    if x.dim() != 2 or x.stride(1) != 1:
        raise VlasrInputError("x must be a 2-D tensor with contiguous rows")
    rows, k = x.shape
    n = w.shape[0]
    if w.dim() != 2 or w.shape[1] != k:
        raise VlasrInputError("w must be [n, k] with x's k")
    cols = n // 2 if epilogue == "swiglu" else n
    if epilogue == "residual":
        if out is None:
            raise VlasrInputError("the residual epilogue updates `out` in place: pass it")
    elif out is None:
        out = torch.empty((rows, cols), dtype=x.dtype, device=x.device)
    _cuda(out, "out")
    _same(x, out, "out")
    if out.dim() != 2 or out.stride(1) != 1 or out.shape != (rows, cols):
        raise VlasrInputError(f"out must be [{rows}, {cols}] with contiguous rows")
    parts = 0
    if norm_weight is not None:
        _contig(norm_weight, "norm_weight")
        _same(x, norm_weight, "norm_weight")
        if ssq_in is None or ssq_in.dtype != torch.float32 or ssq_in.dim() != 2 \
                or ssq_in.shape[1] != rows:
            raise VlasrInputError("the RMSNorm prologue needs ssq_in float32 [parts, rows]")
        _contig(ssq_in, "ssq_in")
        parts = ssq_in.shape[0]
    if ssq_out is not None:
        _contig(ssq_out, "ssq_out")
        if ssq_out.dtype != torch.float32 or ssq_out.shape != (n // 16, rows):
            raise VlasrInputError(f"ssq_out must be float32 [{n // 16}, {rows}]")
    check(_lib.load().vl_decode_linear(
        _ptr(x), x.stride(0), _ptr(norm_weight), _ptr(ssq_in), parts, float(eps), _ptr(w), n, k,
        _ptr(out), out.stride(0), _ptr(ssq_out), rows, LINEAR_EPILOGUES[epilogue],
        _dtype_code(x), (LAUNCH_PDL if pdl else 0) | (LINEAR_TCGEN05 if tcgen05 else 0),
        _stream(x)), "vl_decode_linear")
    return out


# ---------------------------------------------------------------------------
# Decode-step tail
# ---------------------------------------------------------------------------

def argmax_eos(logits: torch.Tensor, *, current: torch.Tensor | None = None,
               finished: torch.Tensor | None = None, row_chunk: torch.Tensor | None = None,
               out: torch.Tensor | None = None, positions: torch.Tensor | None = None,
               prompt_length: torch.Tensor | None = None, eos_ids=(), freeze_id: int = 59253,
               status: torch.Tensor | None = None) -> torch.Tensor:
    """Greedy next token per row with the reference's tie order and EOS
    freeze (vl_argmax_eos).  logits [rows, vocab] (a row stride is allowed).

    Without `finished`: plain argmax per row (current [rows] is returned).
    With finished (bool/uint8 [chunks]), current (int64 [chunks]) and
    optionally row_chunk (int32 [rows]), out (int64 [out_rows, chunks]),
    positions (int32 [chunks]) and prompt_length (int64 device scalar): the
    whole decode-step tail - finished chunks give freeze_id, others store
    their id at out[positions - prompt_length + 1] and finish on an EOS id.
    Returns `current`."""
    _cuda(logits, "logits")
    if logits.dim() != 2 or logits.stride(1) != 1:
        raise VlasrInputError("logits must be a 2-D tensor with contiguous rows")
    rows, vocab = logits.shape
    if row_chunk is not None:
        _contig(row_chunk, "row_chunk")
        if row_chunk.dtype != torch.int32 or row_chunk.numel() != rows:
            raise VlasrInputError("row_chunk must be int32 with one entry per row")
    if current is None:
        if finished is not None or row_chunk is not None:
            raise VlasrInputError("pass `current` (int64 [chunks]) with finished / row_chunk")
        current = torch.empty(rows, dtype=torch.int64, device=logits.device)
    _contig(current, "current")
    if current.dtype != torch.int64 or current.dim() != 1:
        raise VlasrInputError("current must be int64 [chunks]")
    chunks = current.numel()
    if finished is not None:
        _contig(finished, "finished")
        if finished.dtype not in (torch.bool, torch.uint8) or finished.numel() != chunks:
            raise VlasrInputError("finished must be bool/uint8 [chunks]")
    out_rows = out_stride = 0
    if out is not None:
        _contig(out, "out")
        if out.dtype != torch.int64 or out.dim() != 2 or out.shape[1] != chunks:
            raise VlasrInputError("out must be int64 [out_rows, chunks]")
        out_rows, out_stride = out.shape
        for name, t, dt in (("positions", positions, torch.int32),
                            ("prompt_length", prompt_length, torch.int64)):
            if t is None:
                raise VlasrInputError(f"out needs {name}")
            _contig(t, name)
            if t.dtype != dt:
                raise VlasrInputError(f"{name} must be {dt}")
        if positions.numel() != chunks or prompt_length.numel() != 1:
            raise VlasrInputError("positions must be [chunks] and prompt_length a scalar")
    eos = (ctypes.c_int64 * max(len(eos_ids), 1))(*[int(e) for e in eos_ids])
    check(_lib.load().vl_argmax_eos(
        _ptr(logits), rows, vocab, logits.stride(0), _ptr(row_chunk), chunks, _ptr(finished),
        _ptr(current), _ptr(out), out_rows, out_stride, _ptr(positions), _ptr(prompt_length),
        eos, len(eos_ids), int(freeze_id), _dtype_code(logits), _ptr(status),
        _stream(logits)), "vl_argmax_eos")
    return current


# ---------------------------------------------------------------------------
# Index ops
# ---------------------------------------------------------------------------

def embed_gather(ids: torch.Tensor, table: torch.Tensor, *, audio: torch.Tensor | None = None,
                 audio_token_id: int = -1, row_map: torch.Tensor | None = None,
                 shared_ids: bool = False, batch: int | None = None,
                 out: torch.Tensor | None = None,
                 status: torch.Tensor | None = None) -> torch.Tensor:
    """Gather embedding rows for ids [batch, seq] (int64) -> [batch, seq, dim].

    audio [batch, rows, dim] supplies the rows of placeholder ids
    (id == audio_token_id); shared_ids=True uses one id row [seq] for every
    batch entry (the reference's gather_batch_kernel); row_map [batch]
    selects the id row (and audio batch) of each output row.
    """
    _contig(ids, "ids")
    _contig(table, "table")
    if ids.dtype != torch.int64:
        raise VlasrInputError("ids must be int64 (as in the reference)")
    vocab, dim = table.shape
    if shared_ids:
        seq = ids.shape[-1]
        if batch is None:
            batch = audio.shape[0] if audio is not None else 1
        ids_stride = 0
    else:
        if ids.dim() == 1:
            ids2 = ids.view(1, -1)
        else:
            ids2 = ids.view(-1, ids.shape[-1])
        seq = ids2.shape[1]
        ids_stride = seq
        if batch is None:
            batch = ids2.shape[0] if row_map is None else row_map.numel()
    if row_map is not None:
        _contig(row_map, "row_map")
        if row_map.dtype != torch.int32:
            raise VlasrInputError("row_map must be int32")
    audio_rows, audio_stride = 0, 0
    if audio is not None:
        _contig(audio, "audio")
        _same(table, audio, "audio")
        audio_rows = audio.shape[-2]
        audio_stride = audio_rows * dim if audio.dim() == 3 else 0
    if out is None:
        out = torch.empty((batch, seq, dim), dtype=table.dtype, device=table.device)
    _contig(out, "out")
    _same(table, out, "out")
    if out.numel() != batch * seq * dim:
        raise VlasrInputError("out has the wrong size")
    check(_lib.load().vl_embed_gather(_ptr(ids), batch, seq, ids_stride, _ptr(row_map),
                                      _ptr(table), vocab, dim, _ptr(audio), audio_token_id,
                                      audio_rows, audio_stride, _ptr(out), _dtype_code(table),
                                      _ptr(status), _stream(table)), "vl_embed_gather")
    return out


def kv_append(k: torch.Tensor, v: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
              slot_mapping: torch.Tensor, status: torch.Tensor | None = None) -> None:
    """k_cache[slot_mapping[t]] = k[t]; v_cache[...] = v[t] (rows of kv_heads*head_dim)."""
    for name, t in (("k_cache", k_cache), ("v_cache", v_cache), ("slot_mapping", slot_mapping)):
        _contig(t, name)
    _cuda(k, "k")
    _cuda(v, "v")
    _same(k_cache, k, "k")
    _same(k_cache, v, "v")
    if slot_mapping.dtype != torch.int64:
        raise VlasrInputError("slot_mapping must be int64")
    tokens = slot_mapping.numel()
    row = k_cache.shape[-1] * (k_cache.shape[-2] if k_cache.dim() >= 3 else 1)
    kv_heads = k_cache.shape[-2] if k_cache.dim() >= 3 else 1
    head_dim = row // kv_heads
    num_slots = k_cache.numel() // row
    k2, v2 = _rows2d(k, "k", row), _rows2d(v, "v", row)
    if k2.shape[0] != tokens or v2.shape[0] != tokens:
        raise VlasrInputError("k/v must be [tokens, kv_heads*head_dim] with contiguous rows")
    check(_lib.load().vl_kv_append(_ptr(k2), _ptr(v2), _ptr(k_cache), _ptr(v_cache),
                                   _ptr(slot_mapping), tokens, kv_heads, head_dim, k2.stride(0),
                                   v2.stride(0), num_slots, _dtype_code(k_cache), _ptr(status),
                                   _stream(k_cache)), "vl_kv_append")


# ---------------------------------------------------------------------------
# Log-mel frontend
# ---------------------------------------------------------------------------

def logmel_workspace_bytes(chunks: int) -> int:
    return int(_lib.load().vl_logmel_workspace_bytes(chunks))


def logmel(pcm: torch.Tensor, out: torch.Tensor | None = None,
           workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Whisper log-mel features: pcm [chunks, 480000] f32 -> [chunks, 128, 3000] f32."""
    _contig(pcm, "pcm")
    if pcm.dtype != torch.float32:
        raise VlasrInputError("pcm must be float32")
    if pcm.numel() == 0 or pcm.numel() % CHUNK_SAMPLES:
        raise VlasrInputError("pcm must hold chunks * 480000 samples (zero-pad each chunk)")
    chunks = pcm.numel() // CHUNK_SAMPLES
    if out is None:
        out = torch.empty((chunks, MEL_BINS, MEL_FRAMES), dtype=torch.float32, device=pcm.device)
    _contig(out, "out")
    need = logmel_workspace_bytes(chunks)
    if workspace is None:
        workspace = torch.empty(need, dtype=torch.uint8, device=pcm.device)
    _contig(workspace, "workspace")
    check(_lib.load().vl_logmel(_ptr(pcm), chunks, _ptr(out), _ptr(workspace),
                                workspace.numel() * workspace.element_size(), _stream(pcm)),
          "vl_logmel")
    return out
