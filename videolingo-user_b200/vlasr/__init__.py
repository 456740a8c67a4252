"""vlasr - B200 (sm_100a) kernels for the memory-bound layer ops of the
GLM-ASR native engine of VideoLingo-user, behind a C ABI (libvlasr.so).

Importing the package does not touch CUDA; the shared library is loaded on
the first op call (or by `vlasr.load()`), and fails loudly when it is absent.
"""

from ._lib import (VL_BF16, VL_F16, VL_F32, VL_STATUS_BAD_AUDIO, VL_STATUS_BAD_ID,
                   VL_STATUS_BAD_SLOT, SIGNATURES, VlasrError, VlasrExecutionError,
                   VlasrInputError, load)
from .ops import (CHUNK_SAMPLES, MEL_BINS, MEL_FRAMES, add_layernorm, add_rmsnorm,
                  argmax_eos, decode_attention, decode_attention_workspace_bytes, decode_linear,
                  decode_rows,
                  embed_gather, gelu_erf, init,
                  kv_append, logmel, logmel_workspace_bytes, rope_, rope_kv_append, swiglu)

__all__ = [
    "VL_BF16", "VL_F16", "VL_F32", "VL_STATUS_BAD_AUDIO", "VL_STATUS_BAD_ID", "VL_STATUS_BAD_SLOT",
    "SIGNATURES", "VlasrError", "VlasrExecutionError", "VlasrInputError", "load",
    "CHUNK_SAMPLES", "MEL_BINS", "MEL_FRAMES", "add_layernorm", "add_rmsnorm", "argmax_eos",
    "decode_attention", "decode_attention_workspace_bytes", "decode_linear", "decode_rows", "embed_gather",
    "gelu_erf", "init", "kv_append", "logmel", "logmel_workspace_bytes", "rope_", "rope_kv_append",
    "swiglu",
]
