"""GPU: the decode-step linear layer (vl_decode_linear) against a torch fp32
reference of the same math with the reference's rounding points
(native/asr/src/decoder.cu: `gemm` outputs rounded to the storage type,
rmsnorm_kernel, residual_add_kernel, silu_mul_kernel), for every epilogue,
with and without the RMSNorm prologue, at 1..64 token rows - every test
twice: the default (mma.sync) kernel and the opt-in tcgen05 kernel
(VL_LINEAR_TCGEN05)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import vlasr
from helpers import TOL, normwise, to_np

pytestmark = pytest.mark.gpu

DT = [(torch.bfloat16, "bf16"), (torch.float16, "f16")]
_TC = [False]


@pytest.fixture(params=[False, True], ids=["mma_sync", "tcgen05"], autouse=True)
def _kernel(request):
    _TC[0] = request.param
    yield
    _TC[0] = False


def _lin(*args, **kwargs):
    """vl_decode_linear through the kernel this test instance exercises."""
    return vlasr.decode_linear(*args, tcgen05=_TC[0], **kwargs)


def _rand(shape, dev, dtype, seed, std=1.0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(shape, generator=g) * std).to(dtype).to(dev)


def _r(t, dtype):
    return t.to(dtype).float()


def _norm_ref(h, gamma, ssq_rows, k, dtype, eps=1e-5):
    inv = torch.rsqrt(ssq_rows / k + eps)
    return _r(h.float() * inv[:, None] * gamma.float(), dtype)


@pytest.mark.parametrize("dtype,name", DT, ids=["bf16", "f16"])
@pytest.mark.parametrize("rows", [1, 7, 16, 33, 64])
def test_store(dev, dtype, name, rows):
    x = _rand((rows, 2048), dev, dtype, rows)
    w = _rand((3072, 2048), dev, dtype, 100 + rows, 2048 ** -0.5)
    y = _lin(x, w)
    ref = _r(x.float() @ w.float().t(), dtype)
    torch.cuda.synchronize()
    assert normwise(to_np(y), to_np(ref)) <= TOL[name]


@pytest.mark.parametrize("dtype,name", DT, ids=["bf16", "f16"])
def test_swiglu(dev, dtype, name):
    rows, k, ffn = 16, 2048, 6144
    x = _rand((rows, k), dev, dtype, 1)
    w = _rand((2 * ffn, k), dev, dtype, 2, k ** -0.5 * 2)
    y = _lin(x, w, epilogue="swiglu")
    gu = x.float() @ w.float().t()
    g, u = _r(gu[:, :ffn], dtype), _r(gu[:, ffn:], dtype)
    ref = _r(g / (1 + torch.exp(-g)) * u, dtype)
    torch.cuda.synchronize()
    assert y.shape == (rows, ffn)
    assert normwise(to_np(y), to_np(ref)) <= TOL[name]


@pytest.mark.parametrize("dtype,name", DT, ids=["bf16", "f16"])
def test_residual_and_norm_chain(dev, dtype, name):
    """down-projection with the residual epilogue, then a projection whose
    RMSNorm prologue uses the partial sums it produced (a decode layer's
    ffn -> next layer's q|k|v)."""
    rows, hid, ffn = 12, 2048, 6144
    h = _rand((rows, hid), dev, dtype, 3)
    m = _rand((rows, ffn), dev, dtype, 4)
    wd = _rand((hid, ffn), dev, dtype, 5, ffn ** -0.5)
    gamma = _rand(hid, dev, dtype, 6, 0.02) + 1
    wq = _rand((3072, hid), dev, dtype, 7, hid ** -0.5)
    h_ref = _r(h.float() + _r(m.float() @ wd.float().t(), dtype), dtype)
    ssq = torch.empty(hid // 16, rows, dtype=torch.float32, device=dev)
    _lin(m, wd, epilogue="residual", out=h, ssq_out=ssq)
    torch.cuda.synchronize()
    assert normwise(to_np(h), to_np(h_ref)) <= TOL[name]
    # partial sums are exact sums of squares of the new residual values
    hs = h.float().view(rows, hid // 16, 16)
    assert torch.allclose(ssq, (hs * hs).sum(-1).t(), rtol=1e-5, atol=1e-5)
    q = _lin(h, wq, norm_weight=gamma, ssq_in=ssq)
    xn = _norm_ref(h, gamma, (h.float() ** 2).sum(-1), hid, dtype)
    ref = _r(xn @ wq.float().t(), dtype)
    torch.cuda.synchronize()
    assert normwise(to_np(q), to_np(ref)) <= TOL[name]


def test_norm_prologue_matches_add_rmsnorm(dev):
    """RMSNorm prologue == vl_add_rmsnorm then the plain projection."""
    rows, hid = 16, 2048
    h = _rand((rows, hid), dev, torch.bfloat16, 8)
    gamma = _rand(hid, dev, torch.bfloat16, 9, 0.02) + 1
    w = _rand((12288, hid), dev, torch.bfloat16, 10, hid ** -0.5)
    hs = h.float().view(rows, hid // 16, 16)
    ssq = (hs * hs).sum(-1).t().contiguous()
    fused = _lin(h, w, norm_weight=gamma, ssq_in=ssq, epilogue="swiglu")
    xn = vlasr.add_rmsnorm(h.clone(), None, gamma)
    plain = _lin(xn, w, epilogue="swiglu")
    torch.cuda.synchronize()
    same = (fused == plain).float().mean().item()
    assert normwise(to_np(fused), to_np(plain)) <= 1e-2 and same > 0.9, same


def test_row_stride_and_lm_head_width(dev):
    rows, hid, vocab = 5, 2048, 59264
    buf = _rand((rows, 3 * hid), dev, torch.bfloat16, 11)
    x = buf[:, hid:2 * hid]
    w = _rand((vocab, hid), dev, torch.bfloat16, 12, hid ** -0.5)
    y = _lin(x, w)
    ref = _r(x.float() @ w.float().t(), torch.bfloat16)
    torch.cuda.synchronize()
    assert normwise(to_np(y), to_np(ref)) <= TOL["bf16"]
    assert torch.equal(y.float().argmax(-1), ref.argmax(-1)) or \
        normwise(to_np(y), to_np(ref)) < 5e-3


def test_deterministic(dev):
    x = _rand((16, 2048), dev, torch.bfloat16, 13)
    w = _rand((2048, 2048), dev, torch.bfloat16, 14, 2048 ** -0.5)
    a = _lin(x, w)
    b = _lin(x, w)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


def test_rejects(dev):
    x = _rand((65, 2048), dev, torch.bfloat16, 15)
    w = _rand((2048, 2048), dev, torch.bfloat16, 16)
    with pytest.raises(vlasr.VlasrInputError, match="rows"):
        _lin(x, w)
    with pytest.raises(vlasr.VlasrInputError, match="in place"):
        _lin(x[:4], w, epilogue="residual")


def test_pdl_chain_is_bit_identical(dev):
    """VL_LAUNCH_PDL: a decode-layer chain (down + residual -> RMSNorm + q|k|v
    -> RoPE + append + attention -> o + residual -> RMSNorm + gate|up +
    SwiGLU) launched as programmatic dependents gives the same bits as
    ordinary launches, eagerly and replayed from a CUDA graph."""
    rows, hid, ffn, slots = 16, 2048, 6144, 1024
    w_d = _rand((hid, ffn), dev, torch.bfloat16, 20, ffn ** -0.5)
    w_qkv = _rand((3072, hid), dev, torch.bfloat16, 21, hid ** -0.5)
    w_o = _rand((hid, hid), dev, torch.bfloat16, 22, hid ** -0.5)
    w_gu = _rand((2 * ffn, hid), dev, torch.bfloat16, 23, hid ** -0.5)
    g1 = _rand(hid, dev, torch.bfloat16, 24, 0.02) + 1
    g2 = _rand(hid, dev, torch.bfloat16, 25, 0.02) + 1
    h0 = _rand((rows, hid), dev, torch.bfloat16, 26)
    m0 = _rand((rows, ffn), dev, torch.bfloat16, 27)
    kc0 = _rand((rows * slots, 512), dev, torch.bfloat16, 28)
    vc0 = _rand((rows * slots, 512), dev, torch.bfloat16, 29)
    pos = torch.randint(0, 600, (rows,), generator=torch.Generator().manual_seed(30)).to(
        dev, torch.int32)
    start = torch.arange(rows, device=dev, dtype=torch.int64) * slots

    def state():
        return {"h": h0.clone(), "kc": kc0.clone(), "vc": vc0.clone(),
                "sa": torch.empty(128, rows, device=dev), "sb": torch.empty(128, rows, device=dev),
                "ws": torch.zeros(vlasr.decode_attention_workspace_bytes(rows, 16, 4, 128, slots),
                                  dtype=torch.uint8, device=dev),
                "m": torch.empty(rows, ffn, dtype=torch.bfloat16, device=dev)}

    def chain(st, pdl):
        _lin(m0, w_d, epilogue="residual", out=st["h"], ssq_out=st["sa"], pdl=pdl)
        qkv = _lin(st["h"], w_qkv, norm_weight=g1, ssq_in=st["sa"], pdl=pdl)
        a = vlasr.decode_attention(qkv[:, :2048], st["kc"], st["vc"], pos, start, n_kv_heads=4,
                                   head_dim=128, max_seq_len=slots, k=qkv[:, 2048:2560],
                                   v=qkv[:, 2560:], rotary_dim=128, workspace=st["ws"], pdl=pdl)
        _lin(a, w_o, epilogue="residual", out=st["h"], ssq_out=st["sb"], pdl=pdl)
        _lin(st["h"], w_gu, norm_weight=g2, ssq_in=st["sb"], epilogue="swiglu",
                            out=st["m"], pdl=pdl)

    plain, eager = state(), state()
    chain(plain, False)
    chain(eager, True)
    graphed = state()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            chain(graphed, True)
    torch.cuda.current_stream().wait_stream(side)
    graph.replay()
    torch.cuda.synchronize()
    for key in ("h", "m", "kc", "vc", "sa", "sb"):
        assert torch.equal(eager[key], plain[key]), key
        assert torch.equal(graphed[key], plain[key]), key
    del graph


@pytest.mark.parametrize("epilogue,n", [("store", 528), ("store", 16), ("swiglu", 12320),
                                        ("residual", 2064)])
def test_shapes_outside_the_tensor_core_tiles(dev, epilogue, n):
    """Output widths that are not a multiple of 128 columns take the
    mma.sync kernel (the tcgen05 flag is ignored there); same references."""
    rows, k = 9, 2048
    x = _rand((rows, k), dev, torch.bfloat16, 40 + n)
    w = _rand((n, k), dev, torch.bfloat16, 41 + n, k ** -0.5)
    acc = x.float() @ w.float().t()
    if epilogue == "store":
        y = _lin(x, w)
        ref = _r(acc, torch.bfloat16)
    elif epilogue == "swiglu":
        y = _lin(x, w, epilogue="swiglu")
        g, u = _r(acc[:, :n // 2], torch.bfloat16), _r(acc[:, n // 2:], torch.bfloat16)
        ref = _r(g / (1 + torch.exp(-g)) * u, torch.bfloat16)
    else:
        h = _rand((rows, n), dev, torch.bfloat16, 42)
        ref = _r(h.float() + _r(acc, torch.bfloat16), torch.bfloat16)
        y = _lin(x, w, epilogue="residual", out=h)
    torch.cuda.synchronize()
    assert normwise(to_np(y), to_np(ref)) <= TOL["bf16"]


@pytest.mark.parametrize("rows", [1, 16, 17, 32, 33, 64])
def test_tensor_core_row_paddings_all_epilogues(dev, rows):
    """16 / 32 / 64-row MMA tiles (N of the swapped product) at their edges,
    every epilogue, the decoder's widths."""
    hid, ffn = 2048, 6144
    x = _rand((rows, hid), dev, torch.bfloat16, 50 + rows)
    m = _rand((rows, ffn), dev, torch.bfloat16, 51 + rows)
    gamma = _rand(hid, dev, torch.bfloat16, 52, 0.02) + 1
    w_gu = _rand((2 * ffn, hid), dev, torch.bfloat16, 53, hid ** -0.5)
    w_d = _rand((hid, ffn), dev, torch.bfloat16, 54, ffn ** -0.5)
    xs = x.float().view(rows, hid // 16, 16)
    ssq = (xs * xs).sum(-1).t().contiguous()
    y = _lin(x, w_gu, norm_weight=gamma, ssq_in=ssq, epilogue="swiglu")
    xn = _norm_ref(x, gamma, (x.float() ** 2).sum(-1), hid, torch.bfloat16)
    gu = xn @ w_gu.float().t()
    g, u = _r(gu[:, :ffn], torch.bfloat16), _r(gu[:, ffn:], torch.bfloat16)
    ref = _r(g / (1 + torch.exp(-g)) * u, torch.bfloat16)
    h = x.clone()
    part = torch.empty(hid // 16, rows, dtype=torch.float32, device=dev)
    _lin(m, w_d, epilogue="residual", out=h, ssq_out=part)
    h_ref = _r(x.float() + _r(m.float() @ w_d.float().t(), torch.bfloat16), torch.bfloat16)
    torch.cuda.synchronize()
    assert normwise(to_np(y), to_np(ref)) <= TOL["bf16"]
    assert normwise(to_np(h), to_np(h_ref)) <= TOL["bf16"]
    hs = h.float().view(rows, hid // 16, 16)
    assert torch.allclose(part, (hs * hs).sum(-1).t(), rtol=1e-5, atol=1e-5)


def test_zz_no_bounded_wait_expired(dev):
    """Every wait of the tensor-core kernel in this file completed in time."""
    import ctypes
    lib = vlasr.load()
    count = ctypes.c_uint32(12345)
    assert lib.vl_decode_linear_timeouts(ctypes.byref(count)) == 0
    assert count.value == 0
