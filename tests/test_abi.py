"""CPU: the C ABI library loads, exports every symbol include/vl_api.h
declares, and rejects invalid arguments on the host (status 2, message set)
without touching CUDA.  No compute call is made here."""

from __future__ import annotations

import ctypes
import re

import pytest

import vlasr
from conftest import REPO
from vlasr import _lib

HEADER = REPO / "include" / "vl_api.h"


def declared_symbols() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^VL_EXPORT [\w\s\*]+?\b(vl_\w+)\(", text, re.M)))


@pytest.fixture(scope="module")
def lib():
    return vlasr.load()


def test_header_declares_the_expected_ops():
    syms = declared_symbols()
    for name in ("vl_logmel", "vl_add_layernorm", "vl_add_rmsnorm", "vl_gelu_erf", "vl_swiglu",
                 "vl_rope_inplace", "vl_embed_gather", "vl_kv_append", "vl_rope_kv_append",
                 "vl_decode_attention", "vl_decode_attention_workspace_bytes",
                 "vl_decode_linear", "vl_argmax_eos",
                 "vl_last_error", "vl_logmel_workspace_bytes"):
        assert name in syms


def test_library_exports_every_declared_symbol(lib):
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert set(declared_symbols()) == set(_lib.SIGNATURES), "ctypes table out of sync with header"


def test_library_hides_internal_symbols(lib):
    # only the C ABI is exported (built with -fvisibility=hidden)
    with pytest.raises(AttributeError):
        getattr(lib, "_ZN2vl9sm_countEv")


def test_version_and_device_count(lib):
    assert lib.vl_version() >= 100
    assert lib.vl_device_count() >= 0


def test_init_rejects_a_device_that_does_not_exist(lib):
    # no GPU here: every index is out of range; on a GPU box, count is the bound
    n = lib.vl_device_count()
    assert lib.vl_init(n) == _lib.VL_ERR_INVALID
    assert lib.vl_init(-1) == _lib.VL_ERR_INVALID
    assert "vl_init" in lib.vl_last_error().decode()


def test_logmel_workspace_bytes(lib):
    assert lib.vl_logmel_workspace_bytes(0) == 0
    ws1 = lib.vl_logmel_workspace_bytes(1)
    assert ws1 >= 94 * 4 and ws1 % 256 == 0
    assert lib.vl_logmel_workspace_bytes(256) >= 256 * 94 * 4


FAKE = 0x10000  # a 16-byte aligned non-null address; never dereferenced


def _err(lib) -> str:
    return lib.vl_last_error().decode()


@pytest.mark.parametrize("args,needle", [
    ((None, 1, FAKE, FAKE, 1 << 20, None), "null pointer"),
    ((FAKE, 0, FAKE, FAKE, 1 << 20, None), "chunks"),
    ((FAKE + 4, 1, FAKE * 1000, FAKE * 2000, 1 << 20, None), "aligned"),
    ((FAKE, 1, FAKE * 1000, FAKE * 2000, 16, None), "workspace"),
    ((FAKE, 2, FAKE + 480000 * 4, FAKE * 4000, 1 << 20, None), "overlap"),
])
def test_logmel_rejects(lib, args, needle):
    assert lib.vl_logmel(*args) == _lib.VL_ERR_INVALID
    assert needle in _err(lib)


@pytest.mark.parametrize("fn", ["vl_add_layernorm", "vl_add_rmsnorm"])
def test_norm_rejects(lib, fn):
    f = getattr(lib, fn)
    ln = fn == "vl_add_layernorm"

    def call(residual=FAKE, delta=None, w=FAKE * 2, out=FAKE * 3, rows=4, cols=8, eps=1e-5, dtype=2):
        if ln:
            return f(residual, delta, w, None, out, rows, cols, eps, dtype, None)
        return f(residual, delta, w, out, rows, cols, eps, dtype, None)

    assert call(residual=None) == 2 and "null" in _err(lib)
    assert call(w=None) == 2
    assert call(dtype=7) == 2 and "dtype" in _err(lib)
    assert call(cols=0) == 2 and "shape" in _err(lib)
    assert call(rows=-1) == 2
    assert call(eps=float("nan")) == 2 and "eps" in _err(lib)
    assert call(delta=FAKE * 4, out=FAKE) == 2 and "alias" in _err(lib)


def test_gelu_swiglu_reject(lib):
    assert lib.vl_gelu_erf(None, None, FAKE, 1, 8, 2, None) == 2
    assert lib.vl_gelu_erf(FAKE, None, FAKE + 2, 1, 8, 2, None) == 2 and "overlap" in _err(lib)
    assert lib.vl_gelu_erf(FAKE, None, FAKE, 1, 8, 9, None) == 2
    assert lib.vl_swiglu(FAKE, FAKE * 2, FAKE * 3, 2, 8, 4, 8, 8, 2, None) == 2
    assert "stride" in _err(lib)
    assert lib.vl_swiglu(FAKE, None, FAKE * 3, 2, 8, 8, 8, 8, 2, None) == 2


def test_rope_rejects(lib):
    def call(q=FAKE, k=FAKE * 2, tokens=4, nq=16, nk=4, hd=128, rot=64, base=10000.0, qs=2048,
             ks=512, dtype=2, positions=None, row_map=None, pstride=1, seq=0):
        return lib.vl_rope_inplace(q, k, positions, row_map, pstride, 0, tokens, seq, nq, nk, hd,
                                   rot, base, qs, ks, dtype, None)

    assert call(rot=63) == 2 and "rotary_dim" in _err(lib)
    assert call(rot=256, hd=128) == 2
    assert call(rot=0) == 2
    assert call(k=None) == 2 and "n_k_heads" in _err(lib)
    assert call(base=0.0) == 2 and "base" in _err(lib)
    assert call(qs=100) == 2 and "stride" in _err(lib)
    assert call(row_map=FAKE * 5) == 2 and "row_map" in _err(lib)
    assert call(seq=-1) == 2
    assert call(q=None) == 2


def test_index_ops_reject(lib):
    # embed gather: audio substitution without audio rows
    assert lib.vl_embed_gather(FAKE, 1, 4, 4, None, FAKE * 2, 100, 16, None, 99, 3, 0, FAKE * 3, 2,
                               None, None) == 2
    assert "audio" in _err(lib)
    assert lib.vl_embed_gather(FAKE, 1, 4, 4, None, FAKE * 2, 0, 16, None, -1, 0, 0, FAKE * 3, 2,
                               None, None) == 2
    assert lib.vl_kv_append(FAKE, FAKE, FAKE, FAKE, None, 4, 4, 128, 512, 512, 64, 2, None,
                            None) == 2
    assert lib.vl_kv_append(FAKE, FAKE, FAKE, FAKE, FAKE, 4, 4, 128, 100, 512, 64, 2, None,
                            None) == 2
    assert lib.vl_rope_kv_append(FAKE, FAKE * 2, None, FAKE, FAKE, FAKE, FAKE, 4, 16, 4, 128, 64,
                                 10000.0, 64, 2, None, None) == 2


def test_decode_attention_rejects(lib):
    def call(q=FAKE, k=None, v=None, kc=FAKE * 2, vc=FAKE * 3, pos=FAKE * 4, st=FAKE * 5,
             tokens=4, nq=16, nkv=4, hd=128, rot=0, base=10000.0, scale=0.0, qs=2048, ks=512,
             cs=512, max_len=1024, slots=4096, out=FAKE * 6, os_=2048, dtype=2, ws=FAKE * 7,
             ws_bytes=1 << 30, flags=0):
        return lib.vl_decode_attention(q, k, v, kc, vc, pos, st, tokens, nq, nkv, hd, rot, base,
                                       scale, qs, ks, cs, max_len, slots, out, os_, dtype, ws,
                                       ws_bytes, None, flags, None)

    assert call(q=None) == 2 and "null" in _err(lib)
    assert call(k=FAKE * 8) == 2 and "both" in _err(lib)
    assert call(dtype=0) == 2 and "dtype" in _err(lib)
    assert call(nq=14) == 2 and "shape" in _err(lib)
    assert call(hd=96) == 2 and "head_dim" in _err(lib)
    assert call(nq=64, qs=8192, os_=8192) == 2 and "group" in _err(lib)  # 16 per kv head
    assert call(rot=64) == 2 and "RoPE" in _err(lib)            # rotation needs the new k
    assert call(rot=3, k=FAKE * 8, v=FAKE * 9) == 2 and "rotary_dim" in _err(lib)
    assert call(max_len=0) == 2 and "max_seq_len" in _err(lib)
    assert call(max_len=(1 << 18) + 1) == 2
    assert call(cs=256) == 2 and "stride" in _err(lib)
    assert call(qs=2052) == 2 and "multiples of 8" in _err(lib)
    assert call(q=FAKE + 4) == 2 and "aligned" in _err(lib)
    assert call(ws_bytes=16) == 2 and "workspace" in _err(lib)
    assert call(out=FAKE * 2) == 2 and "overlaps" in _err(lib)
    assert call(scale=float("nan")) == 2 and "scale" in _err(lib)
    assert call(flags=2) == 2 and "flags" in _err(lib)
    assert lib.vl_decode_attention_workspace_bytes(64, 16, 4, 128, 4096) >= 64 * 4 * 4
    assert lib.vl_decode_attention_workspace_bytes(0, 16, 4, 128, 4096) == 0
    assert lib.vl_decode_attention_workspace_bytes(1, 16, 3, 128, 4096) == 0


def test_decode_linear_rejects(lib):
    def call(x=FAKE, xs=2048, g=None, ssq=None, parts=0, eps=1e-5, w=FAKE * 2, n=3072, k=2048,
             y=FAKE * 1000, ys=3072, so=None, rows=16, epi=0, dtype=2, flags=0):
        return lib.vl_decode_linear(x, xs, g, ssq, parts, eps, w, n, k, y, ys, so, rows, epi,
                                    dtype, flags, None)

    assert call(x=None) == 2 and "null" in _err(lib)
    assert call(dtype=0) == 2 and "dtype" in _err(lib)
    assert call(epi=7) == 2 and "epilogue" in _err(lib)
    assert call(rows=65) == 2 and "rows" in _err(lib)
    assert call(k=2000, xs=2000) == 2 and "multiple of 512" in _err(lib)
    assert call(n=3000) == 2 and "multiple of 16" in _err(lib)
    assert call(n=3056, epi=1, ys=1528) == 2 and "multiple of 32" in _err(lib)
    assert call(xs=2052) == 2 and "strides" in _err(lib)
    assert call(x=FAKE + 2) == 2 and "aligned" in _err(lib)
    assert call(g=FAKE * 3) == 2 and "ssq_in" in _err(lib)
    assert call(so=FAKE * 4) == 2 and "RESIDUAL" in _err(lib)
    assert call(y=FAKE) == 2 and "overlaps" in _err(lib)
    assert call(flags=4) == 2 and "flags" in _err(lib)
    # VL_LAUNCH_PDL | VL_LINEAR_TCGEN05 are accepted (the next check fails instead)
    assert call(flags=3, rows=65) == 2 and "rows" in _err(lib)
    assert call(g=FAKE * 3 + 4, ssq=FAKE * 4, parts=128) == 2 and "norm_weight" in _err(lib)


def test_argmax_eos_rejects(lib):
    import ctypes
    eos = (ctypes.c_int64 * 3)(59246, 59253, 59255)

    def call(lg=FAKE, rows=16, vocab=59264, rs=59264, rc=None, chunks=16, fin=FAKE * 2,
             cur=FAKE * 3, out=None, out_rows=0, out_stride=0, pos=None, plen=None, n_eos=3,
             dtype=2):
        return lib.vl_argmax_eos(lg, rows, vocab, rs, rc, chunks, fin, cur, out, out_rows,
                                 out_stride, pos, plen, eos, n_eos, 59253, dtype, None, None)

    assert call(lg=None) == 2 and "null" in _err(lib)
    assert call(dtype=5) == 2 and "dtype" in _err(lib)
    assert call(chunks=8) == 2 and "rows" in _err(lib)
    assert call(vocab=59260, rs=59260) == 2 and "vocab" in _err(lib)
    assert call(vocab=1 << 25, rs=1 << 25) == 2 and "vocab" in _err(lib)
    assert call(rs=59268) == 2 and "stride" in _err(lib)
    assert call(lg=FAKE + 8) == 2 and "aligned" in _err(lib)
    assert call(n_eos=9) == 2 and "n_eos" in _err(lib)
    assert call(out=FAKE * 4, out_rows=1024, out_stride=16) == 2 and "positions" in _err(lib)
    assert call(out=FAKE * 4, out_rows=1024, out_stride=8, pos=FAKE * 5, plen=FAKE * 6) == 2
    assert "out_stride" in _err(lib)
    assert call(rows=0, chunks=0) == 0


def test_error_is_thread_local(lib):
    import threading
    assert lib.vl_gelu_erf(None, None, FAKE, 1, 8, 2, None) == 2
    seen = []
    t = threading.Thread(target=lambda: seen.append(lib.vl_last_error()))
    t.start()
    t.join()
    assert seen == [b""]
    assert _err(lib) != ""


def test_status_codes_map_to_exceptions():
    with pytest.raises(vlasr.VlasrInputError):
        _lib.check(_lib.VL_ERR_INVALID, "x")
    with pytest.raises(vlasr.VlasrExecutionError):
        _lib.check(_lib.VL_ERR_EXEC, "x")
    _lib.check(_lib.VL_OK, "x")


def test_ctypes_prototypes_are_complete(lib):
    for name, (restype, argtypes) in _lib.SIGNATURES.items():
        fn = getattr(lib, name)
        assert fn.argtypes == argtypes and fn.restype == restype


def test_missing_library_fails_loudly(tmp_path):
    with pytest.raises(vlasr.VlasrError):
        _lib.load(tmp_path / "nope.so")
    assert isinstance(vlasr.load(), ctypes.CDLL)
