"""GPU: the encoder-layer caller (vlasr.encoder.AudioEncoder) on a synthetic
checkpoint with the full GLM-ASR audio tower, against

* the fp32 restatement (oracle/encoder_ref.py, pinned to transformers), and
* the reference's own engine (load_weights_resident + run_encode_batched,
  compiled from its sources into oracle/_ref) on the same checkpoint and mel.

Float tolerances are normwise relative errors against the fp32 oracle.  A
32-layer stack accumulates the storage rounding of every layer, so the
bounds are looser than the per-op ones, and ours must also be no less
accurate than the reference engine run in its fp32-accumulate mode."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import vlasr
from helpers import normwise, to_np
from oracle.encoder_ref import encode_fp32
from vlasr.checkpoint import load_weights
from vlasr.encoder import AudioEncoder
from vlasr.synth import audio_chunks_device

pytestmark = pytest.mark.gpu

PARTS = ("audio_tower.", "multi_modal_projector.")
CHUNKS = 2
# normwise error bounds against the fp32 oracle after 32 layers
TOL_ENC = {torch.bfloat16: 4e-2, torch.float16: 8e-3}


@pytest.fixture(scope="module")
def ckpt(glmasr_ckpt):
    return glmasr_ckpt


@pytest.fixture(scope="module")
def weights(ckpt, dev):
    _, w = load_weights(ckpt, dev, prefixes=PARTS)
    return w


@pytest.fixture(scope="module")
def mel(dev):
    pcm = audio_chunks_device(CHUNKS, 0, 21, dev)
    return vlasr.logmel(pcm)


@pytest.fixture(scope="module")
def oracle_out(weights, mel):
    return encode_fp32(mel.cpu(), weights, stages=True)


@pytest.fixture(scope="module")
def ours(weights):
    return {dt: AudioEncoder(weights, dtype=dt) for dt in (torch.bfloat16, torch.float16)}


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16], ids=["bf16", "f16"])
def test_encoder_matches_fp32_oracle(ours, mel, oracle_out, dt):
    got = ours[dt].encode(mel, stages=True)
    torch.cuda.synchronize()
    errs = {k: normwise(to_np(got[k]), oracle_out[k].numpy()) for k in got}
    print(f"\nencoder {dt} vs fp32 oracle: {errs}")
    assert got["projector"].shape == (CHUNKS * 375, 2048)
    assert errs["conv_hidden"] <= TOL_ENC[dt] / 4, errs
    assert errs["final_norm"] <= TOL_ENC[dt], errs
    assert errs["projector"] <= TOL_ENC[dt], errs


def test_stage_dumps_do_not_change_the_result(ours, mel):
    enc = ours[torch.bfloat16]
    a = enc.encode(mel, stages=True)["projector"].clone()
    b = enc.encode(mel)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


def test_chunks_are_independent(ours, mel, oracle_out):
    """Encoding chunk 1 alone gives chunk 1's rows of the batched result
    (within GEMM reassociation: cuBLAS may tile M differently)."""
    enc = ours[torch.bfloat16]
    both = enc.encode(mel).clone()
    one = enc.encode(mel[1:2].contiguous())
    torch.cuda.synchronize()
    assert normwise(to_np(one), to_np(both[375:])) <= 1e-2
    assert normwise(to_np(one), oracle_out["projector"][375:].numpy()) <= TOL_ENC[torch.bfloat16]


def test_reduced_layer_stack(weights, mel):
    """`layers=` keeps the first layers only; checked against the oracle at 4."""
    enc = AudioEncoder(weights, dtype=torch.float16, layers=4)
    got = enc.encode(mel[:1].contiguous(), stages=True)
    torch.cuda.synchronize()
    ref = encode_fp32(mel[:1].cpu(), weights, layers=4, stages=True)
    assert normwise(to_np(got["final_norm"]), ref["final_norm"].numpy()) <= 2e-3
    assert normwise(to_np(got["projector"]), ref["projector"].numpy()) <= 2e-3


def test_encoder_rejects_bad_input(ours, dev):
    enc = ours[torch.bfloat16]
    with pytest.raises(vlasr.VlasrInputError):
        enc.encode(torch.zeros(1, 80, 3000, device=dev))
    with pytest.raises(vlasr.VlasrInputError):
        enc.encode(torch.zeros(1, 128, 3000))            # host tensor
    with pytest.raises(vlasr.VlasrInputError):
        enc.encode(torch.zeros(1, 128, 2998, device=dev))  # 1499 frames: not a whole token


def test_encoder_vs_reference_engine(ckpt, ours, mel, oracle_out, ref_kernels, dev):
    lib = ref_kernels
    handle = lib.vlref_load_weights(str(ckpt).encode(), 64 << 30)
    assert handle, lib.vlref_last_error().decode()
    try:
        mel_host = np.ascontiguousarray(to_np(mel))
        ref_out = {}
        for acc in (32, 16):
            out = torch.empty(CHUNKS * 375, 2048, dtype=torch.float16, device=dev)
            torch.cuda.synchronize()
            rc = lib.vlref_encode_batched(handle, mel_host.ctypes.data_as(ctypes.c_void_p), CHUNKS,
                                          int(acc == 16), ctypes.c_void_p(out.data_ptr()))
            assert rc == 0, lib.vlref_last_error().decode()
            torch.cuda.synchronize()
            ref_out[acc] = out
    finally:
        lib.vlref_free_weights(handle)
    want = oracle_out["projector"].numpy()
    err_ref = {acc: normwise(to_np(o), want) for acc, o in ref_out.items()}
    got16 = ours[torch.float16].encode(mel)
    got_bf = ours[torch.bfloat16].encode(mel)
    torch.cuda.synchronize()
    err16 = normwise(to_np(got16), want)
    err_bf = normwise(to_np(got_bf), want)
    vs_ref = normwise(to_np(got16), to_np(ref_out[32]))
    print(f"\nprojector vs fp32 oracle: reference fp32-acc {err_ref[32]:.3e}, reference "
          f"fp16-acc {err_ref[16]:.3e}, ours fp16 {err16:.3e}, ours bf16 {err_bf:.3e}; "
          f"ours fp16 vs reference fp32-acc {vs_ref:.3e}")
    # the reference engine itself is a faithful fp16 implementation ...
    assert err_ref[32] <= TOL_ENC[torch.float16]
    # ... and ours (same storage type) is at least as accurate, and close to it
    assert err16 <= max(1.1 * err_ref[32], 1e-3)
    assert vs_ref <= 2 * TOL_ENC[torch.float16]
