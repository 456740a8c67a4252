"""GPU parity against the reference's OWN kernels.

oracle/_ref/libvlref.so is the reference's native/asr/src/*.cu compiled for
sm_100a from its sources (FP16, the reference's compile-time shapes); each
test runs it and libvlasr on identical seeded inputs.  Index ops must match
bit for bit; float ops within the fp16 tolerance, with the share of
bit-identical outputs reported by the assertion messages.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import vlasr
from helpers import TOL, normwise, to_np
from vlasr.synth import audio_chunks

pytestmark = pytest.mark.gpu

H = torch.float16


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _ok(rc):
    assert rc == 0, f"reference kernel launch failed: CUDA error {rc}"
    torch.cuda.synchronize()


def _rand(shape, dev, seed, mean=0.0, std=1.0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(shape, generator=g) * std + mean).to(H).to(dev)


def test_add_layernorm_vs_reference(dev, ref_kernels):
    rows, cols = 2 * 1500, 1280
    x, d = _rand((rows, cols), dev, 1), _rand((rows, cols), dev, 2)
    w, b = _rand(cols, dev, 3, 1.0, 0.02), _rand(cols, dev, 4, 0.0, 0.02)
    ref_x = x.clone()
    _ok(ref_kernels.vlref_residual_add_enc(_p(ref_x), _p(d), ctypes.c_ulonglong(rows * cols)))
    ref_ln = ref_x.clone()
    _ok(ref_kernels.vlref_layer_norm(_p(ref_ln), _p(w), _p(b), rows, cols))
    out = vlasr.add_layernorm(x, d, w, b)
    torch.cuda.synchronize()
    assert torch.equal(x, ref_x)  # residual: bit-exact
    err = normwise(to_np(out), to_np(ref_ln))
    same = (out == ref_ln).float().mean().item()
    assert err <= TOL["f16"], (err, same)
    assert same > 0.95, same


def test_rmsnorm_vs_reference(dev, ref_kernels):
    rows, cols = 512, 2048
    x, d, w = _rand((rows, cols), dev, 5), _rand((rows, cols), dev, 6), _rand(cols, dev, 7, 1.0, 0.02)
    ref_x = x.clone()
    _ok(ref_kernels.vlref_residual_add_dec(_p(ref_x), _p(d), ctypes.c_ulonglong(rows * cols)))
    ref_n = ref_x.clone()
    _ok(ref_kernels.vlref_rmsnorm(_p(ref_n), _p(w), rows, cols))
    out = vlasr.add_rmsnorm(x, d, w)
    torch.cuda.synchronize()
    assert torch.equal(x, ref_x)
    err = normwise(to_np(out), to_np(ref_n))
    assert err <= TOL["f16"], err


def test_gelu_and_bias_vs_reference(dev, ref_kernels):
    rows, cols = 1500, 5120
    x, b = _rand((rows, cols), dev, 8, 0.0, 2.0), _rand(cols, dev, 9, 0.0, 0.5)
    ref = x.clone()
    _ok(ref_kernels.vlref_add_bias(_p(ref), _p(b), ctypes.c_ulonglong(rows), cols))
    _ok(ref_kernels.vlref_gelu(_p(ref), ctypes.c_ulonglong(rows * cols)))
    out = vlasr.gelu_erf(x, b)
    torch.cuda.synchronize()
    same = (out == ref).float().mean().item()
    assert normwise(to_np(out), to_np(ref)) <= TOL["f16"]
    assert same > 0.999, same


def test_silu_mul_vs_reference(dev, ref_kernels):
    rows, cols = 256, 6144
    g, u = _rand((rows, cols), dev, 10, 0.0, 3.0), _rand((rows, cols), dev, 11)
    ref = g.clone()
    _ok(ref_kernels.vlref_silu_mul(_p(ref), _p(u), ctypes.c_ulonglong(rows * cols)))
    out = vlasr.swiglu(g, u)
    torch.cuda.synchronize()
    same = (out == ref).float().mean().item()
    assert normwise(to_np(out), to_np(ref)) <= TOL["f16"]
    assert same > 0.999, same


def test_encoder_rope_vs_reference(dev, ref_kernels):
    rows = 2 * 1500
    q = _rand((rows, 20 * 64), dev, 12)
    ref = q.clone()
    _ok(ref_kernels.vlref_encoder_rope(_p(ref), rows))
    vlasr.rope_(q.view(rows, 20, 64), None, head_dim=64, rotary_dim=32, seq_len=1500)
    torch.cuda.synchronize()
    same = (q == ref).float().mean().item()
    assert normwise(to_np(q), to_np(ref)) <= TOL["f16"]
    assert same > 0.995, same


def test_decoder_rope_rows_vs_reference(dev, ref_kernels):
    rows, L = 3 * 390, 390
    q, k = _rand((rows, 2048), dev, 13), _rand((rows, 512), dev, 14)
    rq, rk = q.clone(), k.clone()
    _ok(ref_kernels.vlref_rope_rows(_p(rq), _p(rk), rows, L))
    vlasr.rope_(q.view(rows, 16, 128), k.view(rows, 4, 128), head_dim=128, rotary_dim=128,
                seq_len=L)
    torch.cuda.synchronize()
    assert normwise(to_np(q), to_np(rq)) <= TOL["f16"]
    assert normwise(to_np(k), to_np(rk)) <= TOL["f16"]
    assert (q == rq).float().mean().item() > 0.995


def test_decode_rope_map_and_kv_append_vs_reference(dev, ref_kernels):
    chunks, active_n, max_seq = 16, 9, 1024
    rng = np.random.default_rng(15)
    positions = torch.from_numpy(rng.integers(0, max_seq, chunks).astype(np.int32)).to(dev)
    active = torch.from_numpy(rng.permutation(chunks)[:active_n].astype(np.int32)).to(dev)
    q, k, v = _rand((active_n, 2048), dev, 16), _rand((active_n, 512), dev, 17), _rand((active_n, 512), dev, 18)
    rq, rk = q.clone(), k.clone()
    _ok(ref_kernels.vlref_rope_map(_p(rq), _p(rk), _p(positions), _p(active), active_n))
    vlasr.rope_(q.view(active_n, 16, 128), k.view(active_n, 4, 128), head_dim=128,
                rotary_dim=128, positions=positions, row_map=active)
    torch.cuda.synchronize()
    assert normwise(to_np(q), to_np(rq)) <= TOL["f16"]
    assert normwise(to_np(k), to_np(rk)) <= TOL["f16"]
    # KV append: reference cache [chunk][K|V][1024][512] for one layer.
    chunk_stride = 2 * max_seq * 512
    ref_cache = torch.zeros(chunks * chunk_stride, dtype=H, device=dev)
    _ok(ref_kernels.vlref_append_kv_mapped(_p(rk), _p(v), _p(ref_cache),
                                           ctypes.c_void_p(ref_cache.data_ptr() + max_seq * 512 * 2),
                                           _p(positions), _p(active), active_n,
                                           ctypes.c_ulonglong(chunk_stride)))
    ours = torch.zeros_like(ref_cache)
    slot = (active.long() * (chunk_stride // 512) + positions.long()[active.long()])
    kc = ours.view(-1, 512)
    vc = ours[max_seq * 512:].view(-1, 512)[: kc.shape[0] - max_seq]
    # the same K rows on both sides: this checks the index op bit for bit,
    # independently of RoPE's float rounding
    vlasr.kv_append(rk, v, kc, vc, slot)
    torch.cuda.synchronize()
    assert torch.equal(ours.view(torch.int16), ref_cache.view(torch.int16))


def test_gather_batch_and_mapped_vs_reference(dev, ref_kernels):
    rng = np.random.default_rng(19)
    vocab, hidden, L, group, audio_id = 59264, 2048, 400, 3, 59260
    ids = rng.integers(0, 59000, L).astype(np.int64)
    ids[5:380] = audio_id  # 375 audio placeholders, as the GLM-ASR prompt has
    embed = _rand((vocab, hidden), dev, 20, 0.0, 0.02)
    audio = _rand((group, 375, hidden), dev, 21)
    ids_t = torch.from_numpy(ids).to(dev)
    ref = torch.empty(group, L, hidden, dtype=H, device=dev)
    _ok(ref_kernels.vlref_gather_batch(_p(ids_t), L, _p(embed), _p(audio), 375 * hidden, _p(ref),
                                       group))
    out = vlasr.embed_gather(ids_t, embed, audio=audio, audio_token_id=audio_id, shared_ids=True,
                             batch=group)
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
    cur = torch.from_numpy(rng.integers(0, vocab, 20).astype(np.int64)).to(dev)
    act = torch.from_numpy(rng.permutation(20)[:11].astype(np.int32)).to(dev)
    ref2 = torch.empty(11, hidden, dtype=H, device=dev)
    _ok(ref_kernels.vlref_gather_ids_mapped(_p(cur), _p(act), _p(embed), _p(ref2), 11))
    out2 = vlasr.embed_gather(cur.view(20, 1), embed, row_map=act)
    torch.cuda.synchronize()
    assert torch.equal(out2.view(11, hidden).view(torch.int16), ref2.view(torch.int16))


def test_logmel_vs_reference_pipeline(dev, ref_kernels):
    pcm = audio_chunks(2, seed=22)
    ref = np.empty((2, 128, 3000), np.float32)
    rc = ref_kernels.vlref_compute_mel_batched(pcm.ctypes.data_as(ctypes.c_void_p), 2,
                                               ref.ctypes.data_as(ctypes.c_void_p))
    assert rc == 0
    ours = to_np(vlasr.logmel(torch.from_numpy(pcm).to(dev)))
    diff = np.abs(ours.astype(np.float64) - ref)
    assert diff.max() <= 2e-4, diff.max()
    assert normwise(ours, ref) <= 1e-5
