"""CPU oracle for the GLM-ASR layer ops - TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may use
this package, and only as the checker (or the timed CPU baseline); the
product library never imports it.

* The float ops and the reference mel pipeline are a C restatement of the
  reference kernels (vl_oracle.c, loaded through ctypes).  Arrays are numpy
  float32 holding values representable in the storage dtype; results are
  rounded to it.
* `logmel_f64` is the same Whisper log-mel computed in float64 with numpy's
  FFT: the exact-math reference for the normwise tolerance.
* The index ops (gather, KV append) are numpy byte copies.

Parity pins: the mel path is pinned against transformers'
WhisperFeatureExtractor outputs (the reference's own test oracle,
tests/test_native_asr_m0.py:157-190 of VideoLingo-user) stored under
tests/golden/, and against the reference's compiled kernels on the GPU
(oracle/_ref).  The other float ops have no golden vectors in the reference;
they are pinned by tests/golden fixtures generated from the transformers
GLM-ASR modeling semantics and by the reference kernels on the GPU.
"""

from __future__ import annotations

import ctypes
from ctypes import POINTER, c_double, c_float, c_int, c_int64, c_void_p
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"
REF_LIB_PATH = HERE / "_ref" / "libvlref.so"

DTYPE_CODES = {"f32": 0, "f16": 1, "bf16": 2}

_lib = None


def _load():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            from . import build
            build.build_oracle()
        lib = ctypes.CDLL(str(LIB_PATH))
        fp = POINTER(c_float)
        lib.or_round_array.argtypes = [c_int, fp, c_int64]
        lib.or_add_layernorm.argtypes = [fp, c_void_p, fp, c_void_p, fp, c_int64, c_int64, c_float, c_int]
        lib.or_add_rmsnorm.argtypes = [fp, c_void_p, fp, fp, c_int64, c_int64, c_float, c_int]
        lib.or_gelu.argtypes = [fp, c_void_p, fp, c_int64, c_int64, c_int]
        lib.or_swiglu.argtypes = [fp, fp, fp, c_int64, c_int]
        lib.or_rope.argtypes = [fp, fp, POINTER(c_int64), c_int64, c_int, c_int, c_int, c_int,
                                c_double, c_int]
        lib.or_decode_attention.argtypes = [fp, c_void_p, c_void_p, fp, fp, POINTER(ctypes.c_int32),
                                            POINTER(c_int64), c_int64, c_int, c_int, c_int,
                                            c_int, c_double, c_float, c_int, fp]
        lib.or_argmax_eos.argtypes = [fp, c_int64, c_int64, c_void_p, c_void_p,
                                      POINTER(c_int64), c_void_p, c_void_p, c_int64, c_int64,
                                      c_int64, POINTER(c_int64), c_int, c_int64]
        lib.or_mel_filterbank.argtypes = [POINTER(c_double)]
        lib.or_logmel_ref.argtypes = [fp, c_int64, fp]
        for name in ("or_round_array", "or_add_layernorm", "or_add_rmsnorm", "or_gelu",
                     "or_swiglu", "or_rope", "or_mel_filterbank", "or_logmel_ref",
                     "or_decode_attention", "or_argmax_eos"):
            getattr(lib, name).restype = None
        _lib = lib
    return _lib


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _fp(a: np.ndarray):
    return a.ctypes.data_as(POINTER(c_float))


def _opt(a):
    return None if a is None else a.ctypes.data_as(c_void_p)


def round_to(x, dtype: str) -> np.ndarray:
    """Round float32 values to the storage dtype (RNE), returned as float32."""
    y = _f32(x).copy()
    _load().or_round_array(DTYPE_CODES[dtype], _fp(y), y.size)
    return y


def add_layernorm(residual, delta, gamma, beta, eps: float, dtype: str):
    """Returns (new_residual, out), both float32 [rows, cols]."""
    res = _f32(residual).copy()
    cols = res.shape[-1]
    rows = res.size // cols
    d = None if delta is None else _f32(delta)
    g = _f32(gamma)
    b = None if beta is None else _f32(beta)
    out = np.empty_like(res)
    _load().or_add_layernorm(_fp(res), _opt(d), _fp(g), _opt(b), _fp(out), rows, cols, eps,
                             DTYPE_CODES[dtype])
    return res, out


def add_rmsnorm(residual, delta, weight, eps: float, dtype: str):
    res = _f32(residual).copy()
    cols = res.shape[-1]
    rows = res.size // cols
    d = None if delta is None else _f32(delta)
    w = _f32(weight)
    out = np.empty_like(res)
    _load().or_add_rmsnorm(_fp(res), _opt(d), _fp(w), _fp(out), rows, cols, eps,
                           DTYPE_CODES[dtype])
    return res, out


def gelu(x, bias, dtype: str):
    x = _f32(x)
    cols = x.shape[-1]
    rows = x.size // cols
    b = None if bias is None else _f32(bias)
    out = np.empty_like(x)
    _load().or_gelu(_fp(x), _opt(b), _fp(out), rows, cols, DTYPE_CODES[dtype])
    return out


def swiglu(gate, up, dtype: str):
    g, u = _f32(gate), _f32(up)
    out = np.empty_like(g)
    _load().or_swiglu(_fp(g), _fp(u), _fp(out), g.size, DTYPE_CODES[dtype])
    return out


def rope(q, k, positions, head_dim: int, rotary_dim: int, base: float, dtype: str):
    """q [tokens, nq, head_dim], k [tokens, nk, head_dim]; returns rotated copies."""
    qq = _f32(q).copy()
    kk = _f32(k).copy() if k is not None else np.zeros((qq.shape[0], 0, head_dim), np.float32)
    tokens = qq.shape[0]
    pos = np.ascontiguousarray(positions, dtype=np.int64)
    _load().or_rope(_fp(qq), _fp(kk), pos.ctypes.data_as(POINTER(c_int64)), tokens,
                    qq.shape[1], kk.shape[1], head_dim, rotary_dim, base, DTYPE_CODES[dtype])
    return qq, (kk if k is not None else None)


def decode_attention(q, k_cache, v_cache, positions, seq_start, *, k=None, v=None,
                     rotary_dim: int = 0, base: float = 10000.0, scale: float | None = None,
                     dtype: str = "bf16"):
    """Decode step: q [tokens, nq, hd]; caches [num_slots, nkv, hd] (copies are
    updated with the new rows when k/v are given).  Returns (out [tokens, nq,
    hd], k_cache', v_cache')."""
    qq = _f32(q).copy()
    tokens, nq, hd = qq.shape
    kc = _f32(k_cache).copy()
    vc = _f32(v_cache).copy()
    nkv = kc.shape[1]
    kk = _f32(k).copy() if k is not None else None
    vv = _f32(v).copy() if v is not None else None
    pos = np.ascontiguousarray(positions, dtype=np.int32)
    st = np.ascontiguousarray(seq_start, dtype=np.int64)
    out = np.empty((tokens, nq, hd), dtype=np.float32)
    sc = float(1.0 / np.sqrt(hd)) if scale is None else float(scale)
    _load().or_decode_attention(
        _fp(qq), None if kk is None else kk.ctypes.data_as(c_void_p),
        None if vv is None else vv.ctypes.data_as(c_void_p), _fp(kc), _fp(vc),
        pos.ctypes.data_as(POINTER(ctypes.c_int32)), st.ctypes.data_as(POINTER(c_int64)),
        tokens, nq, nkv, hd, rotary_dim, base, sc, DTYPE_CODES[dtype], _fp(out))
    return out, kc, vc


def argmax_eos(logits, *, row_chunk=None, finished=None, current=None, out=None,
               positions=None, prompt_length: int = 0, eos_ids=(), freeze_id: int = 59253):
    """The reference's decode-step argmax (argmax_mapped_kernel; without
    `finished`, argmax_rows_kernel).  logits [rows, vocab] (values of the
    storage type); finished (uint8/bool [chunks]), current (int64 [chunks])
    and out (int64 [out_rows, chunks]) are copied and returned updated:
    (current, finished, out)."""
    lg = _f32(logits)
    rows, vocab = lg.shape
    rc = None if row_chunk is None else np.ascontiguousarray(row_chunk, dtype=np.int32)
    chunks = rows if rc is None else (int(rc.max()) + 1 if rows else 0)
    if current is None:
        cur = np.zeros(chunks, dtype=np.int64)
    else:
        cur = np.ascontiguousarray(current, dtype=np.int64).copy()
    fin = None if finished is None else np.ascontiguousarray(finished, dtype=np.uint8).copy()
    oo = None if out is None else np.ascontiguousarray(out, dtype=np.int64).copy()
    pos = None if positions is None else np.ascontiguousarray(positions, dtype=np.int32)
    eos = np.ascontiguousarray(list(eos_ids) or [0], dtype=np.int64)
    _load().or_argmax_eos(
        _fp(lg), rows, vocab, None if rc is None else rc.ctypes.data_as(c_void_p),
        None if fin is None else fin.ctypes.data_as(c_void_p), cur.ctypes.data_as(POINTER(c_int64)),
        None if oo is None else oo.ctypes.data_as(c_void_p),
        None if pos is None else pos.ctypes.data_as(c_void_p), int(prompt_length),
        0 if oo is None else oo.shape[0], 0 if oo is None else oo.shape[1],
        eos.ctypes.data_as(POINTER(c_int64)), len(eos_ids), int(freeze_id))
    return cur, fin, oo


def mel_filterbank_f64() -> np.ndarray:
    fb = np.empty((201, 128), dtype=np.float64)
    _load().or_mel_filterbank(fb.ctypes.data_as(POINTER(c_double)))
    return fb


def logmel_ref(pcm) -> np.ndarray:
    """The reference's own fp32 mel pipeline restated in C: [C, 480000] -> [C, 128, 3000]."""
    x = _f32(pcm).reshape(-1, 480000)
    out = np.empty((x.shape[0], 128, 3000), dtype=np.float32)
    _load().or_logmel_ref(_fp(x), x.shape[0], _fp(out))
    return out


def logmel_f64(pcm) -> np.ndarray:
    """Exact-math Whisper log-mel in float64 (numpy rfft): [C, 480000] -> [C, 128, 3000]."""
    x = np.asarray(pcm, dtype=np.float64).reshape(-1, 480000)
    n = np.arange(400)
    window = 0.5 * (1.0 - np.cos(2.0 * np.pi * n / 400))
    fb = mel_filterbank_f64()  # [201, 128]
    outs = []
    for chunk in x:
        padded = np.pad(chunk, (200, 200), mode="reflect")
        idx = np.arange(3000)[:, None] * 160 + n[None, :]
        frames = padded[idx] * window[None, :]
        power = np.abs(np.fft.rfft(frames, axis=1)) ** 2  # [3000, 201]
        mel = power @ fb                                   # [3000, 128]
        log = np.log10(np.maximum(mel, 1e-10)).T           # [128, 3000]
        log = np.maximum(log, log.max() - 8.0)
        outs.append((log + 4.0) / 4.0)
    return np.stack(outs)


def embed_gather(ids, table, audio=None, audio_token_id: int = -1, shared_ids: bool = False,
                 batch: int | None = None, row_map=None):
    """Numpy restatement of the gather kernels (decoder.cu:60-78,460-469,636-667).

    Returns (out, status_bits).  Rows are copied as raw bytes (bit-exact)."""
    ids = np.asarray(ids, dtype=np.int64)
    table = np.asarray(table)
    vocab, dim = table.shape
    id_rows = ids.reshape(1, -1) if (shared_ids or ids.ndim == 1) else ids.reshape(-1, ids.shape[-1])
    seq = id_rows.shape[1]
    if batch is None:
        batch = (audio.shape[0] if (shared_ids and audio is not None) else
                 (len(row_map) if row_map is not None else id_rows.shape[0]))
    out = np.zeros((batch, seq, dim), dtype=table.dtype)
    status = 0
    for b in range(batch):
        src = int(row_map[b]) if row_map is not None else b
        row_ids = id_rows[0] if shared_ids else id_rows[src]
        seen = 0
        for s in range(seq):
            i = int(row_ids[s])
            if audio_token_id >= 0 and i == audio_token_id:
                if audio is not None and seen < audio.shape[-2]:
                    out[b, s] = audio[src][seen] if audio.ndim == 3 else audio[seen]
                else:
                    status |= 2
                seen += 1
            elif 0 <= i < vocab:
                out[b, s] = table[i]
            else:
                status |= 1
    return out, status


def kv_append(k, v, k_cache, v_cache, slot_mapping):
    """Numpy restatement of the slot-mapped KV append; returns (k_cache, v_cache, status)."""
    kc, vc = np.array(k_cache, copy=True), np.array(v_cache, copy=True)
    rows = kc.reshape(kc.shape[0], -1).shape[0]
    kc2, vc2 = kc.reshape(rows, -1), vc.reshape(rows, -1)
    k2, v2 = np.asarray(k).reshape(len(slot_mapping), -1), np.asarray(v).reshape(len(slot_mapping), -1)
    status = 0
    for t, slot in enumerate(np.asarray(slot_mapping, dtype=np.int64)):
        if slot < 0:
            continue
        if slot >= rows:
            status |= 4
            continue
        kc2[slot] = k2[t]
        vc2[slot] = v2[t]
    return kc, vc, status


def load_reference_kernels():
    """ctypes handle of oracle/_ref/libvlref.so (the reference's CUDA kernels), or None."""
    if not REF_LIB_PATH.exists():
        return None
    lib = ctypes.CDLL(str(REF_LIB_PATH))
    # the engine entry points (ref_harness/ref_encoder.cu) return pointers
    lib.vlref_last_error.restype = ctypes.c_char_p
    lib.vlref_load_weights.restype = c_void_p
    lib.vlref_load_weights.argtypes = [ctypes.c_char_p, ctypes.c_ulonglong]
    lib.vlref_free_weights.restype = None
    lib.vlref_free_weights.argtypes = [c_void_p]
    lib.vlref_weights_bytes.restype = ctypes.c_ulonglong
    lib.vlref_weights_bytes.argtypes = [c_void_p]
    lib.vlref_encode_batched.restype = c_int
    lib.vlref_encode_batched.argtypes = [c_void_p, c_void_p, c_int, c_int, c_void_p]
    lib.vlref_decode_batched.restype = c_int
    lib.vlref_decode_batched.argtypes = [c_void_p, c_void_p, c_int, c_void_p, c_int, c_int, c_int,
                                         c_void_p, c_void_p, c_void_p, c_void_p]
    return lib
