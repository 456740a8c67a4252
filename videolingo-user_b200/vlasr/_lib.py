"""ctypes binding of libvlasr.so (the C ABI in include/vl_api.h).

The library is loaded once, from this package directory.  A missing or
unloadable library raises immediately: there is no fallback implementation.
Status codes map onto the reference engine's error taxonomy
(native/asr/src/model_loader.h:14-25): 2 -> VlasrInputError (ModelInputError),
1 -> VlasrExecutionError (ModelExecutionError).
"""

from __future__ import annotations

import ctypes
import threading
from ctypes import c_double, c_float, c_int, c_int64, c_size_t, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libvlasr.so"

VL_OK, VL_ERR_EXEC, VL_ERR_INVALID = 0, 1, 2
VL_F32, VL_F16, VL_BF16 = 0, 1, 2
VL_STATUS_BAD_ID, VL_STATUS_BAD_AUDIO, VL_STATUS_BAD_SLOT = 1, 2, 4
VL_IPC_HANDLE_BYTES = 64

# Every symbol the header declares, with (restype, argtypes).
SIGNATURES = {
    "vl_version": (c_int, []),
    "vl_last_error": (ctypes.c_char_p, []),
    "vl_device_count": (c_int, []),
    "vl_init": (c_int, [c_int]),
    "vl_ipc_export": (c_int, [c_void_p, c_void_p, ctypes.POINTER(ctypes.c_uint64)]),
    "vl_ipc_open": (c_int, [c_void_p, ctypes.POINTER(c_void_p)]),
    "vl_ipc_close": (c_int, [c_void_p]),
    "vl_copy_async": (c_int, [c_void_p, c_void_p, c_size_t, c_void_p]),
    "vl_logmel_workspace_bytes": (c_size_t, [c_int64]),
    "vl_logmel": (c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_size_t, c_void_p]),
    "vl_logmel_noalloc": (c_int, [c_void_p, c_int64, c_void_p, c_void_p]),
    "vl_add_layernorm": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64,
                                 c_int64, c_float, c_int, c_void_p]),
    "vl_add_rmsnorm": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_float,
                               c_int, c_void_p]),
    "vl_gelu_erf": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int, c_void_p]),
    "vl_swiglu": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64,
                          c_int64, c_int, c_void_p]),
    "vl_rope_inplace": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64,
                                c_int64, c_int, c_int, c_int, c_int, c_double, c_int64, c_int64,
                                c_int, c_void_p]),
    "vl_embed_gather": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_int64,
                                c_int64, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int,
                                c_void_p, c_void_p]),
    "vl_kv_append": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int,
                             c_int, c_int64, c_int64, c_int64, c_int, c_void_p, c_void_p]),
    "vl_rope_kv_append": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                  c_void_p, c_int64, c_int, c_int, c_int, c_int, c_double, c_int64,
                                  c_int, c_void_p, c_void_p]),
    "vl_decode_rows": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_float,
                               c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                               c_void_p, c_int64, c_int, c_int, c_int, c_int, c_double, c_int64,
                               c_int64, c_int64, c_int, c_void_p, c_void_p]),
    "vl_decode_attention_workspace_bytes": (c_size_t, [c_int64, c_int, c_int, c_int, c_int64]),
    "vl_decode_linear": (c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_int, c_float, c_void_p,
                                 c_int64, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_int,
                                 c_int, c_int, c_void_p]),
    "vl_decode_linear_timeouts": (c_int, [ctypes.POINTER(ctypes.c_uint32)]),
    "vl_argmax_eos": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_void_p,
                              c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_void_p,
                              ctypes.POINTER(c_int64), c_int, c_int64, c_int, c_void_p,
                              c_void_p]),
    "vl_decode_attention": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                    c_void_p, c_int64, c_int, c_int, c_int, c_int, c_double,
                                    c_float, c_int64, c_int64, c_int64, c_int64, c_int64,
                                    c_void_p, c_int64, c_int, c_void_p, c_size_t, c_void_p,
                                    c_int, c_void_p]),
}


class VlasrError(RuntimeError):
    """Base class of library failures."""


class VlasrInputError(VlasrError, ValueError):
    """Invalid argument (status 2; the reference's ModelInputError)."""


class VlasrExecutionError(VlasrError):
    """CUDA launch/execution failure (status 1; the reference's ModelExecutionError)."""


_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load(path: Path | str | None = None) -> ctypes.CDLL:
    """Load libvlasr.so (once) and attach the prototypes."""
    global _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        target = Path(path) if path is not None else LIB_PATH
        if not target.exists():
            raise VlasrError(
                f"{target} is missing: build it with `python -m vlasr.build` "
                "(there is no CPU fallback for these ops)")
        lib = ctypes.CDLL(str(target))
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        if path is None:
            _lib = lib
        return lib


def check(status: int, op: str) -> None:
    if status == VL_OK:
        return
    msg = (load().vl_last_error() or b"").decode(errors="replace") or op
    if status == VL_ERR_INVALID:
        raise VlasrInputError(msg)
    raise VlasrExecutionError(msg)
