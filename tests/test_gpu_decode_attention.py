"""GPU parity of the decode-step attention (vl_decode_attention) against the
C oracle (oracle/vl_oracle.c or_decode_attention, a restatement of the
reference's rope_at_position_map + append_kv_mapped +
attention_step_mapped kernels) and against those reference kernels
compiled from their sources (oracle/_ref).

Float outputs: normwise relative error within the storage type's tolerance.
Cache rows written without RoPE are bit-exact copies."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import oracle
import vlasr
from helpers import TOL, normwise, to_np

pytestmark = pytest.mark.gpu

NQ, NKV, HD = 16, 4, 128


def _rand(shape, dev, dtype, seed, std=1.0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(shape, generator=g) * std).to(dtype).to(dev)


def _setup(dev, dtype, seqs, slots_per_seq, seed, positions=None):
    rng = np.random.default_rng(seed)
    pos = positions if positions is not None else rng.integers(0, slots_per_seq, seqs)
    pos = torch.tensor(np.asarray(pos, np.int32), device=dev)
    start = torch.arange(seqs, device=dev, dtype=torch.int64) * slots_per_seq
    q = _rand((seqs, NQ * HD), dev, dtype, seed + 1)
    k = _rand((seqs, NKV * HD), dev, dtype, seed + 2)
    v = _rand((seqs, NKV * HD), dev, dtype, seed + 3)
    kc = _rand((seqs * slots_per_seq, NKV * HD), dev, dtype, seed + 4)
    vc = _rand((seqs * slots_per_seq, NKV * HD), dev, dtype, seed + 5)
    return q, k, v, kc, vc, pos, start


def _oracle(q, kc, vc, pos, start, k=None, v=None, rot=0, dtype="bf16"):
    t = q.shape[0]
    out, kc2, vc2 = oracle.decode_attention(
        to_np(q).reshape(t, NQ, HD), to_np(kc).reshape(-1, NKV, HD), to_np(vc).reshape(-1, NKV, HD),
        pos.cpu().numpy(), start.cpu().numpy(),
        k=None if k is None else to_np(k).reshape(t, NKV, HD),
        v=None if v is None else to_np(v).reshape(t, NKV, HD), rotary_dim=rot, dtype=dtype)
    return out.reshape(t, NQ * HD), kc2.reshape(-1, NKV * HD), vc2.reshape(-1, NKV * HD)


DT = [(torch.bfloat16, "bf16"), (torch.float16, "f16")]


@pytest.mark.parametrize("dtype,name", DT, ids=["bf16", "f16"])
@pytest.mark.parametrize("fused", [False, True], ids=["cache_only", "rope_append"])
def test_decode_attention_vs_oracle(dev, dtype, name, fused):
    q, k, v, kc, vc, pos, start = _setup(dev, dtype, 24, 1024, seed=10)
    kc0, vc0 = kc.clone(), vc.clone()
    if fused:
        out = vlasr.decode_attention(q, kc, vc, pos, start, n_kv_heads=NKV, head_dim=HD, k=k, v=v,
                                     rotary_dim=HD, max_seq_len=1024)
        want, kw, vw = _oracle(q, kc0, vc0, pos, start, k, v, rot=HD, dtype=name)
    else:
        out = vlasr.decode_attention(q, kc, vc, pos, start, n_kv_heads=NKV, head_dim=HD,
                                     max_seq_len=1024)
        want, kw, vw = _oracle(q, kc0, vc0, pos, start, dtype=name)
    torch.cuda.synchronize()
    assert normwise(to_np(out), want) <= TOL[name]
    if fused:
        # appended rows: rotated k (fp32 cos/sin of the reduced fp64 angle vs
        # the oracle's fp64 cos/sin rounded: ties may flip), v copied
        slots = (start + pos.long()).cpu().numpy()
        assert normwise(to_np(kc)[slots], kw[slots]) <= TOL[name]
        assert np.array_equal(to_np(vc)[slots], vw[slots])
        untouched = np.ones(kc.shape[0], bool)
        untouched[slots] = False
        assert torch.equal(kc[torch.from_numpy(untouched).to(dev)],
                           kc0[torch.from_numpy(untouched).to(dev)])
    else:
        assert torch.equal(kc, kc0) and torch.equal(vc, vc0)


def test_append_without_rope_is_a_copy(dev):
    q, k, v, kc, vc, pos, start = _setup(dev, torch.bfloat16, 8, 256, seed=20)
    vlasr.decode_attention(q, kc, vc, pos, start, n_kv_heads=NKV, head_dim=HD, k=k, v=v,
                           max_seq_len=256)
    torch.cuda.synchronize()
    slots = start + pos.long()
    assert torch.equal(kc[slots], k) and torch.equal(vc[slots], v)


@pytest.mark.parametrize("p", [0, 1, 63, 64, 65, 511, 512, 513, 1023])
def test_split_boundaries(dev, p):
    """Single-token calls (the split heuristic gives 64-position splits) at
    lengths around the split edges; the fused and the unfused path agree."""
    q, k, v, kc, vc, pos, start = _setup(dev, torch.float16, 1, 1024, seed=30 + p, positions=[p])
    kc0, vc0 = kc.clone(), vc.clone()
    out = vlasr.decode_attention(q, kc, vc, pos, start, n_kv_heads=NKV, head_dim=HD, k=k, v=v,
                                 rotary_dim=HD, max_seq_len=1024)
    want, _, _ = _oracle(q, kc0, vc0, pos, start, k, v, rot=HD, dtype="f16")
    torch.cuda.synchronize()
    assert normwise(to_np(out), want) <= TOL["f16"]


def test_config3_shape_against_torch_fp32(dev):
    """64 sequences x 4096 slots, positions U[0, 4096) (the decode benchmark
    configuration) against a torch fp32 reference of the same attention."""
    q, k, v, kc, vc, pos, start = _setup(dev, torch.bfloat16, 64, 4096, seed=40)
    out = vlasr.decode_attention(q, kc, vc, pos, start, n_kv_heads=NKV, head_dim=HD,
                                 max_seq_len=4096)
    torch.cuda.synchronize()
    ref = torch.empty(64, NQ, HD, device=dev)
    for t in range(64):
        n = int(pos[t]) + 1
        s0 = int(start[t])
        K = kc[s0:s0 + n].float().view(n, NKV, HD).repeat_interleave(NQ // NKV, dim=1)
        V = vc[s0:s0 + n].float().view(n, NKV, HD).repeat_interleave(NQ // NKV, dim=1)
        qq = q[t].float().view(NQ, HD)
        sc = torch.einsum("hd,nhd->hn", qq, K) / HD ** 0.5
        ref[t] = torch.einsum("hn,nhd->hd", torch.softmax(sc, -1), V)
    assert normwise(to_np(out), to_np(ref.view(64, -1))) <= TOL["bf16"]


def test_workspace_is_left_zero_and_calls_repeat(dev):
    q, k, v, kc, vc, pos, start = _setup(dev, torch.bfloat16, 16, 2048, seed=50)
    nbytes = vlasr.decode_attention_workspace_bytes(16, NQ, NKV, HD, 2048)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
    a = vlasr.decode_attention(q, kc, vc, pos, start, n_kv_heads=NKV, head_dim=HD,
                               max_seq_len=2048, workspace=ws)
    b = vlasr.decode_attention(q, kc, vc, pos, start, n_kv_heads=NKV, head_dim=HD,
                               max_seq_len=2048, workspace=ws)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert int(ws[:16 * NKV * 4].count_nonzero()) == 0  # split counters reset


def test_bad_positions_and_slots(dev):
    q, k, v, kc, vc, pos, start = _setup(dev, torch.bfloat16, 6, 128, seed=60)
    pos[1] = 128          # >= max_seq_len
    pos[3] = -1
    start[4] = 6 * 128 - 2  # start + pos beyond the cache for pos >= 2
    pos[4] = 5
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    kc0 = kc.clone()
    out = vlasr.decode_attention(q, kc, vc, pos, start, n_kv_heads=NKV, head_dim=HD, k=k, v=v,
                                 rotary_dim=HD, max_seq_len=128, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & vlasr.VL_STATUS_BAD_SLOT
    for t in (1, 3, 4):
        assert int(out[t].count_nonzero()) == 0
    good = [0, 2, 5]
    want, _, _ = _oracle(q[good], kc0, vc.clone(), pos[good], start[good], k[good], v[good],
                         rot=HD)
    assert normwise(to_np(out[good]), want) <= TOL["bf16"]


def test_rows_of_a_packed_qkv_buffer(dev):
    """q / k / v as column slices of one packed [tokens, (16+4+4)*128] buffer."""
    q, k, v, kc, vc, pos, start = _setup(dev, torch.bfloat16, 8, 512, seed=70)
    qkv = torch.cat([q, k, v], 1)
    kc0, vc0 = kc.clone(), vc.clone()
    out = vlasr.decode_attention(qkv[:, :NQ * HD], kc, vc, pos, start, n_kv_heads=NKV,
                                 head_dim=HD, k=qkv[:, NQ * HD:(NQ + NKV) * HD],
                                 v=qkv[:, (NQ + NKV) * HD:], rotary_dim=HD, max_seq_len=512)
    want, _, _ = _oracle(q, kc0, vc0, pos, start, k, v, rot=HD)
    torch.cuda.synchronize()
    assert normwise(to_np(out), want) <= TOL["bf16"]


@pytest.mark.parametrize("nq,nkv,hd", [(8, 8, 128), (8, 4, 128), (16, 2, 128), (16, 2, 64),
                                       (8, 8, 64), (32, 8, 64)])
def test_other_head_groupings(dev, nq, nkv, hd):
    rng = np.random.default_rng(80)
    T, L = 5, 300
    pos = torch.tensor(rng.integers(0, L, T).astype(np.int32), device=dev)
    start = torch.arange(T, device=dev, dtype=torch.int64) * L
    q = _rand((T, nq * hd), dev, torch.float16, 81)
    kc = _rand((T * L, nkv * hd), dev, torch.float16, 82)
    vc = _rand((T * L, nkv * hd), dev, torch.float16, 83)
    out = vlasr.decode_attention(q, kc, vc, pos, start, n_kv_heads=nkv, head_dim=hd,
                                 max_seq_len=L)
    want, _, _ = oracle.decode_attention(
        to_np(q).reshape(T, nq, hd), to_np(kc).reshape(-1, nkv, hd),
        to_np(vc).reshape(-1, nkv, hd), pos.cpu().numpy(), start.cpu().numpy(), dtype="f16")
    torch.cuda.synchronize()
    assert normwise(to_np(out), want.reshape(T, -1)) <= TOL["f16"]


def test_rejects(dev):
    q, k, v, kc, vc, pos, start = _setup(dev, torch.bfloat16, 2, 64, seed=90)
    with pytest.raises(vlasr.VlasrInputError, match="head_dim"):
        vlasr.decode_attention(q, kc, vc, pos, start, n_kv_heads=2, head_dim=256, max_seq_len=64)
    with pytest.raises(vlasr.VlasrInputError):
        vlasr.decode_attention(q, kc, vc, pos, start, n_kv_heads=NKV, head_dim=HD, k=k,
                               max_seq_len=64)
    with pytest.raises(vlasr.VlasrInputError, match="RoPE"):
        vlasr.decode_attention(q, kc, vc, pos, start, n_kv_heads=NKV, head_dim=HD, rotary_dim=HD,
                               max_seq_len=64)


# ---------------------------------------------------------------------------
# against the reference's own kernels (FP16, <= 1024 positions)
# ---------------------------------------------------------------------------

def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def test_vs_reference_decode_kernels(dev, ref_kernels):
    lib = ref_kernels
    chunks, rows, max_seq = 12, 9, 1024
    rng = np.random.default_rng(100)
    positions = torch.from_numpy(rng.integers(0, max_seq, chunks).astype(np.int32)).to(dev)
    active = torch.from_numpy(rng.permutation(chunks)[:rows].astype(np.int32)).to(dev)
    h = torch.float16
    q = _rand((rows, NQ * HD), dev, h, 101)
    k = _rand((rows, NKV * HD), dev, h, 102)
    v = _rand((rows, NKV * HD), dev, h, 103)
    chunk_stride = 2 * max_seq * NKV * HD          # one layer: [K|V][1024][512]
    cache = _rand((chunks * chunk_stride,), dev, h, 104)
    # reference: rope at positions[active[r]], append, attention
    rq, rk, rcache = q.clone(), k.clone(), cache.clone()
    assert lib.vlref_rope_map(_p(rq), _p(rk), _p(positions), _p(active), rows) == 0
    vbase = ctypes.c_void_p(rcache.data_ptr() + max_seq * NKV * HD * 2)
    assert lib.vlref_append_kv_mapped(_p(rk), _p(v), _p(rcache), vbase, _p(positions),
                                      _p(active), rows, ctypes.c_ulonglong(chunk_stride)) == 0
    rout = torch.empty(rows, NQ * HD, dtype=h, device=dev)
    assert lib.vlref_attention_mapped(_p(rq), _p(rcache), _p(rout), _p(positions), _p(active),
                                      rows, 0, ctypes.c_ulonglong(0),
                                      ctypes.c_ulonglong(chunk_stride)) == 0
    torch.cuda.synchronize()
    # ours: one fused call on the same layout (K rows of chunk c start at
    # slot c*2048, V rows 1024 slots later)
    ours_cache = cache.clone()
    nrows = ours_cache.numel() // (NKV * HD) - max_seq
    kview = ours_cache.view(-1, NKV * HD)[:nrows]
    vview = ours_cache[max_seq * NKV * HD:].view(-1, NKV * HD)[:nrows]
    act = active.long()
    seq_start = act * (chunk_stride // (NKV * HD))
    row_pos = positions[act].contiguous()
    out = vlasr.decode_attention(q, kview, vview, row_pos, seq_start, n_kv_heads=NKV, head_dim=HD,
                                 k=k, v=v, rotary_dim=HD, max_seq_len=max_seq)
    torch.cuda.synchronize()
    err = normwise(to_np(out), to_np(rout))
    same = (out == rout).float().mean().item()
    assert err <= TOL["f16"], (err, same)
    # appended V rows are identical; K rows within rounding of the rotation
    slots = (seq_start + row_pos.long())
    assert torch.equal(vview[slots], rcache[max_seq * NKV * HD:].view(-1, NKV * HD)[slots])
    kk = kview[slots]
    rkk = rcache.view(-1, NKV * HD)[slots]
    assert normwise(to_np(kk), to_np(rkk)) <= TOL["f16"]
    assert (kk == rkk).float().mean().item() > 0.99
