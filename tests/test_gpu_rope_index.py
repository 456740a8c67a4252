"""GPU parity: RoPE (every position mode of the reference), embedding gather
and KV append (bit-exact), and the fused decode-step RoPE + KV append."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
import vlasr
from helpers import TOL, from_np, normwise, to_np, torch_dtype

pytestmark = pytest.mark.gpu


def _qk(tokens, nq, nk, hd, dtype, seed):
    rng = np.random.default_rng(seed)
    q = oracle.round_to(rng.normal(0, 1, (tokens, nq, hd)), dtype)
    k = oracle.round_to(rng.normal(0, 1, (tokens, nk, hd)), dtype)
    return q, k


@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("tokens,nq,nk,hd,rot", [
    (3000, 20, 20, 64, 32),     # encoder: partial rotary 32 of 64, pos = row % 1500
    (256, 16, 4, 128, 64),      # decoder config: first half of 128
    (33, 16, 4, 128, 128),      # reference decoder: full rotary
    (5, 2, 1, 40, 20),          # rotary half not a multiple of 8 -> scalar path
    (7, 3, 0, 64, 64),          # q only
])
def test_rope_row_positions(dev, dtype, tokens, nq, nk, hd, rot):
    seq_len = 1500 if hd == 64 and rot == 32 else 0
    q, k = _qk(tokens, nq, nk, hd, dtype, seed=tokens + rot)
    td = torch_dtype(dtype)
    qt = from_np(q, td, dev)
    kt = from_np(k, td, dev) if nk else None
    vlasr.rope_(qt, kt, head_dim=hd, rotary_dim=rot, seq_len=seq_len)
    pos = np.arange(tokens) % seq_len if seq_len else np.arange(tokens)
    eq, ek = oracle.rope(q, k if nk else None, pos, hd, rot, 10000.0, dtype)
    assert normwise(to_np(qt), eq) <= TOL[dtype]
    np.testing.assert_array_equal(to_np(qt)[..., rot:], q[..., rot:])
    if nk:
        assert normwise(to_np(kt), ek) <= TOL[dtype]


def test_rope_prefill_config_full_size(dev):
    """Config 2: Q [4,2048,16,128], K [4,2048,4,128] bf16, rotary 64, positions 0..2047."""
    q, k = _qk(4 * 2048, 16, 4, 128, "bf16", seed=21)
    qt, kt = from_np(q, torch.bfloat16, dev), from_np(k, torch.bfloat16, dev)
    vlasr.rope_(qt.view(4, 2048, 16, 128), kt.view(4, 2048, 4, 128), head_dim=128, rotary_dim=64,
                seq_len=2048)
    pos = np.arange(4 * 2048) % 2048
    eq, ek = oracle.rope(q, k, pos, 128, 64, 10000.0, "bf16")
    gq, gk = to_np(qt), to_np(kt)
    assert normwise(gq, eq) <= TOL["bf16"] and normwise(gk, ek) <= TOL["bf16"]
    assert (gq == eq).mean() > 0.99 and (gk == ek).mean() > 0.99


def test_rope_scattered_positions_row_map_and_scalar(dev):
    """Decode modes: per-row positions through an active-row map, a shared
    device scalar (stride 0) and a host scalar (seq_len 1 + offset)."""
    q, k = _qk(64, 16, 4, 128, "bf16", seed=31)
    rng = np.random.default_rng(32)
    positions = rng.integers(0, 4096, 100).astype(np.int32)
    active = rng.permutation(100)[:64].astype(np.int32)
    td = torch.bfloat16
    qt, kt = from_np(q, td, dev), from_np(k, td, dev)
    vlasr.rope_(qt, kt, head_dim=128, rotary_dim=64,
                positions=torch.from_numpy(positions).to(dev),
                row_map=torch.from_numpy(active).to(dev))
    eq, ek = oracle.rope(q, k, positions[active], 128, 64, 10000.0, "bf16")
    assert normwise(to_np(qt), eq) <= TOL["bf16"] and normwise(to_np(kt), ek) <= TOL["bf16"]

    qt, kt = from_np(q, td, dev), from_np(k, td, dev)
    vlasr.rope_(qt, kt, head_dim=128, rotary_dim=128,
                positions=torch.tensor([777], dtype=torch.int32, device=dev), positions_stride=0)
    eq, ek = oracle.rope(q, k, np.full(64, 777), 128, 128, 10000.0, "bf16")
    assert normwise(to_np(qt), eq) <= TOL["bf16"] and normwise(to_np(kt), ek) <= TOL["bf16"]

    qt, kt = from_np(q, td, dev), from_np(k, td, dev)
    vlasr.rope_(qt, kt, head_dim=128, rotary_dim=128, seq_len=1, pos_offset=391)
    eq, ek = oracle.rope(q, k, np.full(64, 391), 128, 128, 10000.0, "bf16")
    assert normwise(to_np(qt), eq) <= TOL["bf16"] and normwise(to_np(kt), ek) <= TOL["bf16"]


def test_rope_packed_qkv_row_strides(dev):
    """q and k as views into one packed [tokens, (16+4+4)*128] QKV buffer."""
    rng = np.random.default_rng(41)
    tokens = 50
    qkv = oracle.round_to(rng.normal(0, 1, (tokens, 24 * 128)), "bf16")
    buf = from_np(qkv, torch.bfloat16, dev)
    qv = buf[:, :2048].view(tokens, 16, 128)
    kv = buf[:, 2048:2560].view(tokens, 4, 128)
    vlasr.rope_(qv, kv, head_dim=128, rotary_dim=64)
    eq, ek = oracle.rope(qkv[:, :2048].reshape(tokens, 16, 128),
                         qkv[:, 2048:2560].reshape(tokens, 4, 128), np.arange(tokens), 128, 64,
                         10000.0, "bf16")
    got = to_np(buf)
    assert normwise(got[:, :2048].reshape(tokens, 16, 128), eq) <= TOL["bf16"]
    assert normwise(got[:, 2048:2560].reshape(tokens, 4, 128), ek) <= TOL["bf16"]
    np.testing.assert_array_equal(got[:, 2560:], qkv[:, 2560:])  # V untouched


# ---------------------------------------------------------------------------
# Index ops: bit-exact
# ---------------------------------------------------------------------------

def _bits(t: torch.Tensor) -> np.ndarray:
    return t.view(torch.int16 if t.element_size() == 2 else torch.int32).cpu().numpy()


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("dim", [2048, 1280, 7, 100])
def test_embed_gather_plain(dev, dtype, dim):
    rng = np.random.default_rng(dim)
    vocab = 5000
    table = from_np(rng.normal(0, 0.02, (vocab, dim)), torch_dtype(dtype), dev)
    ids = rng.integers(0, vocab, (3, 17)).astype(np.int64)
    out = vlasr.embed_gather(torch.from_numpy(ids).to(dev), table)
    exp = table[torch.from_numpy(ids).to(dev)]
    np.testing.assert_array_equal(_bits(out), _bits(exp))


def test_embed_gather_prefill_config_full_size(dev):
    """Config 2: ids U[0,151552) [4, 2048] int64 from a [151552, 2048] bf16 table."""
    g = torch.Generator(device="cpu").manual_seed(7)
    table = (torch.randn(151552, 2048, generator=g) * 0.02).to(torch.bfloat16).to(dev)
    ids = torch.randint(0, 151552, (4, 2048), generator=g, dtype=torch.int64).to(dev)
    out = vlasr.embed_gather(ids, table)
    np.testing.assert_array_equal(_bits(out), _bits(table[ids]))


def test_embed_gather_audio_placeholders_shared_prompt(dev):
    """gather_batch semantics: one prompt shared by every chunk, placeholder
    rows taken from each chunk's own projector rows in order."""
    rng = np.random.default_rng(5)
    vocab, dim, L, chunks, audio_rows, audio_id = 300, 64, 40, 3, 12, 299
    ids = rng.integers(0, 290, L).astype(np.int64)
    ids[[2, 3, 4, 10, 11, 30]] = audio_id
    table = rng.normal(0, 1, (vocab, dim)).astype(np.float32)
    audio = rng.normal(0, 1, (chunks, audio_rows, dim)).astype(np.float32)
    t_tab = from_np(table, torch.bfloat16, dev)
    t_aud = from_np(audio, torch.bfloat16, dev)
    out = vlasr.embed_gather(torch.from_numpy(ids).to(dev), t_tab, audio=t_aud,
                             audio_token_id=audio_id, shared_ids=True, batch=chunks)
    exp, status = oracle.embed_gather(ids, to_np(t_tab), audio=to_np(t_aud),
                                      audio_token_id=audio_id, shared_ids=True, batch=chunks)
    assert status == 0
    np.testing.assert_array_equal(to_np(out), exp)


def test_embed_gather_row_map_and_bad_ids(dev):
    rng = np.random.default_rng(6)
    vocab, dim = 100, 32
    table = from_np(rng.normal(0, 1, (vocab, dim)), torch.float32, dev)
    ids = torch.from_numpy(rng.integers(0, vocab, (10, 1)).astype(np.int64)).to(dev)
    ids[3, 0] = -5
    ids[7, 0] = vocab
    active = torch.tensor([9, 3, 0, 7], dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    out = vlasr.embed_gather(ids, table, row_map=active, status=status)
    exp, st = oracle.embed_gather(ids.cpu().numpy(), table.cpu().numpy(),
                                  row_map=active.cpu().numpy())
    np.testing.assert_array_equal(to_np(out), exp)
    assert int(status.item()) == st == vlasr.VL_STATUS_BAD_ID
    assert not to_np(out)[1].any() and not to_np(out)[3].any()


def test_embed_gather_too_many_placeholders(dev):
    ids = torch.tensor([[5, 9, 9, 9]], dtype=torch.int64, device=dev)
    table = torch.arange(10 * 8, dtype=torch.float32, device=dev).view(10, 8)
    audio = torch.ones(1, 2, 8, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    out = vlasr.embed_gather(ids, table, audio=audio, audio_token_id=9, status=status)
    assert int(status.item()) == vlasr.VL_STATUS_BAD_AUDIO
    got = to_np(out)[0]
    np.testing.assert_array_equal(got[0], np.arange(40, 48))
    assert (got[1:3] == 1).all() and not got[3].any()


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_kv_append_slot_mapping(dev, dtype):
    """Config 3: 64 tokens, 4 KV heads x 128, 64 x 4096 slots, distinct seeded slots;
    -1 skips, an out-of-range slot is skipped and flagged."""
    rng = np.random.default_rng(8)
    tokens, heads, hd, slots = 64, 4, 128, 64 * 4096
    td = torch_dtype(dtype)
    k = from_np(rng.normal(0, 1, (tokens, heads, hd)), td, dev)
    v = from_np(rng.normal(0, 1, (tokens, heads, hd)), td, dev)
    kc = torch.zeros(slots, heads, hd, dtype=td, device=dev)
    vc = torch.zeros_like(kc)
    slot = (np.arange(64) * 4096 + rng.integers(0, 4096, 64)).astype(np.int64)
    slot[5] = -1
    slot[9] = slots + 3
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    vlasr.kv_append(k, v, kc, vc, torch.from_numpy(slot).to(dev), status=status)
    assert int(status.item()) == vlasr.VL_STATUS_BAD_SLOT
    ok = (slot >= 0) & (slot < slots)
    idx = torch.from_numpy(slot[ok]).to(dev)
    np.testing.assert_array_equal(_bits(kc[idx]), _bits(k[torch.from_numpy(ok).to(dev)]))
    np.testing.assert_array_equal(_bits(vc[idx]), _bits(v[torch.from_numpy(ok).to(dev)]))
    assert int((kc != 0).any(-1).any(-1).sum().item()) == int(ok.sum())


def test_kv_append_many_tokens_warp_path(dev):
    """Above 2 tokens per SM the append runs one warp per token (prefill)."""
    rng = np.random.default_rng(12)
    tokens, slots = 1000, 4096
    k = from_np(rng.normal(0, 1, (tokens, 4, 128)), torch.bfloat16, dev)
    v = from_np(rng.normal(0, 1, (tokens, 4, 128)), torch.bfloat16, dev)
    kc = torch.zeros(slots, 4, 128, dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    slot = torch.from_numpy(rng.permutation(slots)[:tokens].astype(np.int64)).to(dev)
    vlasr.kv_append(k, v, kc, vc, slot)
    np.testing.assert_array_equal(_bits(kc[slot]), _bits(k))
    np.testing.assert_array_equal(_bits(vc[slot]), _bits(v))


def test_kv_append_strided_rows(dev):
    """K/V as column slices of a packed QKV buffer (row stride > row width)."""
    rng = np.random.default_rng(9)
    tokens = 10
    qkv = from_np(rng.normal(0, 1, (tokens, 24 * 128)), torch.bfloat16, dev)
    k, v = qkv[:, 2048:2560], qkv[:, 2560:3072]
    kc = torch.zeros(32, 4, 128, dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    slot = torch.arange(tokens, dtype=torch.int64, device=dev) * 3
    vlasr.kv_append(k, v, kc, vc, slot)
    np.testing.assert_array_equal(_bits(kc[slot].view(tokens, -1)), _bits(k))
    np.testing.assert_array_equal(_bits(vc[slot].view(tokens, -1)), _bits(v))


def test_rope_kv_append_matches_separate_ops(dev):
    rng = np.random.default_rng(10)
    tokens, slots = 64, 64 * 4096
    q, k = _qk(tokens, 16, 4, 128, "bf16", seed=11)
    v = oracle.round_to(rng.normal(0, 1, (tokens, 4, 128)), "bf16")
    pos = rng.integers(0, 4096, tokens).astype(np.int32)
    slot = (np.arange(tokens) * 4096 + pos).astype(np.int64)
    slot[3] = -1
    td = torch.bfloat16
    q1, k1, v1 = from_np(q, td, dev), from_np(k, td, dev), from_np(v, td, dev)
    kc1 = torch.zeros(slots, 4, 128, dtype=td, device=dev)
    vc1 = torch.zeros_like(kc1)
    pos_t, slot_t = torch.from_numpy(pos).to(dev), torch.from_numpy(slot).to(dev)
    vlasr.rope_kv_append(q1, k1, v1, kc1, vc1, pos_t, slot_t, head_dim=128, rotary_dim=64)
    q2, k2 = from_np(q, td, dev), from_np(k, td, dev)
    kc2, vc2 = torch.zeros_like(kc1), torch.zeros_like(kc1)
    vlasr.rope_(q2, k2, head_dim=128, rotary_dim=64, positions=pos_t)
    vlasr.kv_append(k2, from_np(v, td, dev), kc2, vc2, slot_t)
    for a, b in ((q1, q2), (k1, k2), (kc1, kc2), (vc1, vc2)):
        np.testing.assert_array_equal(_bits(a), _bits(b))
    eq, ek = oracle.rope(q, k, pos, 128, 64, 10000.0, "bf16")
    assert normwise(to_np(q1), eq) <= TOL["bf16"] and normwise(to_np(k1), ek) <= TOL["bf16"]


@pytest.mark.parametrize("dtype,tokens,nq,nk,hd,rot", [
    ("bf16", 1001, 16, 4, 128, 64),    # config-2 heads, partial last token group
    ("f32", 3000, 20, 20, 64, 32),     # encoder heads, fp32 (2 vectors per half)
    ("f16", 700, 16, 4, 128, 128),     # full rotary (8 vectors per half)
    ("f32", 400, 16, 4, 128, 128),     # fp32 full rotary (16 vectors per half)
    ("bf16", 333, 3, 1, 64, 64),       # few heads: several tokens per block group
])
def test_rope_inplace_matches_fused_append_at_stream_sizes(dev, dtype, tokens, nq, nk, hd, rot):
    """vl_rope_inplace and vl_rope_kv_append at prefill-like token counts
    (persistent warps, several tokens each, partial last round) must give
    the same bits for q and k, and match the oracle."""
    rng = np.random.default_rng(tokens + rot)
    q, k = _qk(tokens, nq, nk, hd, dtype, seed=tokens)
    v = oracle.round_to(rng.normal(0, 1, (tokens, nk, hd)), dtype)
    pos = (rng.integers(0, 4096, tokens)).astype(np.int32)
    td = torch_dtype(dtype)
    q1, k1 = from_np(q, td, dev), from_np(k, td, dev)
    pos_t = torch.from_numpy(pos).to(dev)
    vlasr.rope_(q1, k1, head_dim=hd, rotary_dim=rot, positions=pos_t)
    q2, k2, v2 = from_np(q, td, dev), from_np(k, td, dev), from_np(v, td, dev)
    kc = torch.zeros(tokens, nk, hd, dtype=td, device=dev)
    vc = torch.zeros_like(kc)
    slot = torch.arange(tokens, dtype=torch.int64, device=dev)
    vlasr.rope_kv_append(q2, k2, v2, kc, vc, pos_t, slot, head_dim=hd, rotary_dim=rot)
    np.testing.assert_array_equal(_bits(q1), _bits(q2))
    np.testing.assert_array_equal(_bits(k1), _bits(k2))
    eq, ek = oracle.rope(q, k, pos, hd, rot, 10000.0, dtype)
    assert normwise(to_np(q1), eq) <= TOL[dtype] and normwise(to_np(k1), ek) <= TOL[dtype]
    np.testing.assert_array_equal(to_np(q1)[..., rot:], q[..., rot:])
