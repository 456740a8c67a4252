"""GPU parity of vl_decode_rows: the row ops of a decode step in one launch
(residual add + RMSNorm of the hidden rows; RoPE of q/k at each position
with the KV append), against the CPU oracle and against the ops' own entry
points (vl_add_rmsnorm, vl_rope_kv_append) on the same inputs.

The norm part runs the same block-per-row routine as vl_add_rmsnorm on few
rows, so its outputs must be bit-identical; the appended cache rows must be
bit-identical to the rotated k and to v."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
import vlasr
from helpers import TOL, from_np, normwise, to_np, torch_dtype

pytestmark = pytest.mark.gpu


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.view(torch.int16 if t.element_size() == 2 else torch.int32).cpu().numpy()


def _case(dtype, rows, cols, tokens, nq, nk, hd, slots, seed):
    rng = np.random.default_rng(seed)
    r = lambda *s: oracle.round_to(rng.normal(0, 1, s), dtype)  # noqa: E731
    res, delta = r(rows, cols), r(rows, cols)
    w = oracle.round_to(rng.normal(1, 0.02, cols), dtype)
    q, k, v = r(tokens, nq, hd), r(tokens, nk, hd), r(tokens, nk, hd)
    pos = rng.integers(0, 4096, tokens).astype(np.int32)
    slot = rng.permutation(slots)[:tokens].astype(np.int64)
    return res, delta, w, q, k, v, pos, slot


def _run(dev, dtype, case, *, with_delta=True, rot=64, slots=None):
    res, delta, w, q, k, v, pos, slot = case
    td = torch_dtype(dtype)
    tokens, nq, hd = q.shape
    nk = k.shape[1]
    t = {"res": from_np(res, td, dev), "delta": from_np(delta, td, dev),
         "w": from_np(w, td, dev), "q": from_np(q.reshape(tokens, -1), td, dev),
         "k": from_np(k.reshape(tokens, -1), td, dev), "v": from_np(v.reshape(tokens, -1), td, dev),
         "kc": torch.zeros(slots, nk, hd, dtype=td, device=dev),
         "pos": torch.from_numpy(pos).to(dev), "slot": torch.from_numpy(slot).to(dev),
         "status": torch.zeros(1, dtype=torch.int32, device=dev)}
    t["vc"] = torch.zeros_like(t["kc"])
    t["out"] = vlasr.decode_rows(t["res"], t["delta"] if with_delta else None, t["w"], t["q"],
                                 t["k"], t["v"], t["kc"], t["vc"], t["pos"], t["slot"],
                                 head_dim=hd, rotary_dim=rot, status=t["status"])
    torch.cuda.synchronize()
    return t


@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("with_delta", [True, False])
def test_decode_rows_config3_matches_oracle(dev, dtype, with_delta):
    """Config 3: 64 rows of 2048; Q [64,16,128], K/V [64,4,128], rotary 64,
    positions U[0,4096), distinct slots of a 64 x 4096-slot cache."""
    slots = 64 * 4096
    case = _case(dtype, 64, 2048, 64, 16, 4, 128, slots, seed=3)
    res, delta, w, q, k, v, pos, slot = case
    t = _run(dev, dtype, case, with_delta=with_delta, slots=slots)
    exp_res, exp_out = oracle.add_rmsnorm(res, delta if with_delta else None, w, 1e-5, dtype)
    np.testing.assert_array_equal(to_np(t["res"]), exp_res)
    assert normwise(to_np(t["out"]), exp_out) <= TOL[dtype]
    eq, ek = oracle.rope(q, k, pos, 128, 64, 10000.0, dtype)
    gq, gk = to_np(t["q"]).reshape(q.shape), to_np(t["k"]).reshape(k.shape)
    assert normwise(gq, eq) <= TOL[dtype] and normwise(gk, ek) <= TOL[dtype]
    np.testing.assert_array_equal(gq[..., 64:], q[..., 64:])
    idx = t["slot"]
    np.testing.assert_array_equal(_bits(t["kc"][idx].reshape(64, -1)), _bits(t["k"]))
    np.testing.assert_array_equal(_bits(t["vc"][idx].reshape(64, -1)), _bits(t["v"]))
    assert int(t["status"].item()) == 0
    assert int((t["kc"] != 0).any(-1).any(-1).sum().item()) == 64


def test_decode_rows_equals_separate_entry_points(dev):
    """Same inputs through vl_add_rmsnorm and vl_rope_kv_append: the norm
    outputs and the appended rows are bit-identical; q/k agree to rounding."""
    slots = 64 * 4096
    case = _case("bf16", 64, 2048, 64, 16, 4, 128, slots, seed=4)
    res, delta, w, q, k, v, pos, slot = case
    t = _run(dev, "bf16", case, slots=slots)
    td = torch.bfloat16
    r2, d2, w2 = from_np(res, td, dev), from_np(delta, td, dev), from_np(w, td, dev)
    out2 = vlasr.add_rmsnorm(r2, d2, w2)
    q2, k2, v2 = (from_np(a.reshape(64, -1), td, dev) for a in (q, k, v))
    kc2 = torch.zeros(slots, 4, 128, dtype=td, device=dev)
    vc2 = torch.zeros_like(kc2)
    vlasr.rope_kv_append(q2, k2, v2, kc2, vc2, t["pos"], t["slot"], head_dim=128, rotary_dim=64)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(_bits(t["out"]), _bits(out2))
    np.testing.assert_array_equal(_bits(t["res"]), _bits(r2))
    np.testing.assert_array_equal(_bits(t["vc"]), _bits(vc2))
    for a, b in ((t["q"], q2), (t["k"], k2), (t["kc"], kc2)):
        ga, gb = to_np(a), to_np(b)
        assert normwise(ga, gb) <= 1e-3
        assert (ga == gb).mean() > 0.999


@pytest.mark.parametrize("nq,nk,hd,rot", [(16, 4, 128, 128), (8, 2, 64, 32), (32, 8, 128, 64)])
def test_decode_rows_head_shapes(dev, nq, nk, hd, rot):
    """Full and partial rotary, other head counts; 32+8 heads x 128 with rot
    64 has more tasks per token than threads (the block loops)."""
    slots = 4096
    case = _case("bf16", 16, 1024, 24, nq, nk, hd, slots, seed=nq + hd + rot)
    res, delta, w, q, k, v, pos, slot = case
    t = _run(dev, "bf16", case, rot=rot, slots=slots)
    _, exp_out = oracle.add_rmsnorm(res, delta, w, 1e-5, "bf16")
    assert normwise(to_np(t["out"]), exp_out) <= TOL["bf16"]
    eq, ek = oracle.rope(q, k, pos, hd, rot, 10000.0, "bf16")
    assert normwise(to_np(t["q"]).reshape(q.shape), eq) <= TOL["bf16"]
    assert normwise(to_np(t["k"]).reshape(k.shape), ek) <= TOL["bf16"]
    idx = t["slot"]
    np.testing.assert_array_equal(_bits(t["kc"][idx].reshape(24, -1)), _bits(t["k"]))
    np.testing.assert_array_equal(_bits(t["vc"][idx].reshape(24, -1)), _bits(t["v"]))


def test_decode_rows_bad_and_skipped_slots(dev):
    slots = 512
    case = list(_case("bf16", 4, 2048, 8, 16, 4, 128, slots, seed=9))
    slot = case[7].copy()
    slot[2] = -1
    slot[5] = slots + 7
    case[7] = slot
    t = _run(dev, "bf16", tuple(case), slots=slots)
    assert int(t["status"].item()) == vlasr.VL_STATUS_BAD_SLOT
    eq, ek = oracle.rope(case[3], case[4], case[6], 128, 64, 10000.0, "bf16")
    assert normwise(to_np(t["q"]).reshape(eq.shape), eq) <= TOL["bf16"]  # every q still rotates
    assert int((t["kc"] != 0).any(-1).any(-1).sum().item()) == 6


def test_decode_rows_one_part_only(dev):
    """rows = 0 or tokens = 0: the launch does only the other part."""
    slots = 256
    case = _case("bf16", 8, 2048, 8, 16, 4, 128, slots, seed=13)
    res, delta, w, q, k, v, pos, slot = case
    td = torch.bfloat16
    empty = torch.empty(0, 2048, dtype=td, device=dev)
    qt, kt, vt = (from_np(a.reshape(8, -1), td, dev) for a in (q, k, v))
    kc = torch.zeros(slots, 4, 128, dtype=td, device=dev)
    vc = torch.zeros_like(kc)
    vlasr.decode_rows(empty, None, from_np(w, td, dev), qt, kt, vt, kc, vc,
                      torch.from_numpy(pos).to(dev), torch.from_numpy(slot).to(dev),
                      head_dim=128, rotary_dim=64)
    rt = from_np(res, td, dev)
    q0 = torch.empty(0, 2048, dtype=td, device=dev)
    k0 = torch.empty(0, 512, dtype=td, device=dev)
    out = vlasr.decode_rows(rt, from_np(delta, td, dev), from_np(w, td, dev), q0, k0, k0, kc, vc,
                            torch.empty(0, dtype=torch.int32, device=dev),
                            torch.empty(0, dtype=torch.int64, device=dev), head_dim=128)
    torch.cuda.synchronize()
    eq, _ = oracle.rope(q, k, pos, 128, 64, 10000.0, "bf16")
    assert normwise(to_np(qt).reshape(eq.shape), eq) <= TOL["bf16"]
    _, exp_out = oracle.add_rmsnorm(res, delta, w, 1e-5, "bf16")
    assert normwise(to_np(out), exp_out) <= TOL["bf16"]


def test_decode_rows_rejects_overlap_and_misalignment(dev):
    td = torch.bfloat16
    flat = torch.zeros(16 * 2048, dtype=td, device=dev)
    rows = flat[:8 * 2048].view(8, 2048)
    w = torch.ones(2048, dtype=td, device=dev)
    kc = torch.zeros(64, 4, 128, dtype=td, device=dev)
    pos = torch.zeros(8, dtype=torch.int32, device=dev)
    slot = torch.arange(8, dtype=torch.int64, device=dev)
    k = torch.zeros(8, 512, dtype=td, device=dev)
    # q shares its first half with the norm rows
    q_alias = flat[4 * 2048:12 * 2048].view(8, 2048)
    with pytest.raises(vlasr.VlasrInputError, match="overlap"):
        vlasr.decode_rows(rows, None, w, q_alias, k, k.clone(), kc, kc.clone(), pos, slot,
                          head_dim=128)
    q = torch.zeros(8, 2048, dtype=td, device=dev)
    with pytest.raises(vlasr.VlasrInputError, match="multiples"):
        vlasr.decode_rows(rows, None, w, q, k, k.clone(), kc, kc.clone(), pos, slot,
                          head_dim=128, rotary_dim=12)
