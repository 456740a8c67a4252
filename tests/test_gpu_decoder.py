"""GPU: the text decoder (vlasr.decoder.TextDecoder) and the in-process engine
(vlasr.engine.AsrEngine) against the reference's own batched decode
(run_decode_batched, compiled from its sources into oracle/_ref) on the same
synthetic checkpoint, projector rows and prompt.

Greedy decoding of a random-weight model is compared by teacher forcing: our
decoder is fed the reference's tokens and must pick the reference's next
token at every step, except where its own top-1 / top-2 logits are closer
than the rounding noise of the two fp16 pipelines (a near tie)."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import vlasr
from vlasr.checkpoint import load_weights
from vlasr.decoder import AUDIO_TOKEN_ID, EOS_IDS, TextDecoder
from vlasr.encoder import AudioEncoder
from vlasr.engine import AsrEngine
from vlasr.synth import audio_chunks_device

pytestmark = pytest.mark.gpu

CHUNKS = 3
NEW = 24
PROMPT = [151, 2222, 3333] + [AUDIO_TOKEN_ID] * 375 + [4444, 5555, 6666, 77]
NEAR_TIE = 0.15  # logits; fp16 storage + different GEMM orders differ by ~1e-2


@pytest.fixture(scope="module")
def weights(glmasr_ckpt, dev):
    _, w = load_weights(glmasr_ckpt, dev)
    return w


@pytest.fixture(scope="module")
def audio16(weights, dev):
    mel = vlasr.logmel(audio_chunks_device(CHUNKS, 0, 31, dev))
    return AudioEncoder(weights, dtype=torch.float16).encode(mel).contiguous()


@pytest.fixture(scope="module")
def reference_ids(glmasr_ckpt, audio16, ref_kernels):
    lib = ref_kernels
    handle = lib.vlref_load_weights(str(glmasr_ckpt).encode(), 64 << 30)
    assert handle, lib.vlref_last_error().decode()
    try:
        prompt = np.asarray(PROMPT, np.int64)
        out = np.full((CHUNKS, NEW), -1, np.int64)
        lens = np.zeros(CHUNKS, np.int32)
        pre, dec = ctypes.c_float(), ctypes.c_float()
        torch.cuda.synchronize()
        rc = lib.vlref_decode_batched(handle, ctypes.c_void_p(audio16.data_ptr()), CHUNKS,
                                      prompt.ctypes.data_as(ctypes.c_void_p), len(PROMPT), NEW,
                                      0, out.ctypes.data_as(ctypes.c_void_p),
                                      lens.ctypes.data_as(ctypes.c_void_p), ctypes.byref(pre),
                                      ctypes.byref(dec))
        assert rc == 0, lib.vlref_last_error().decode()
    finally:
        lib.vlref_free_weights(handle)
    return [out[c, :lens[c]].tolist() for c in range(CHUNKS)]


@pytest.fixture(scope="module")
def decoders(weights):
    return {dt: TextDecoder(weights, dtype=dt) for dt in (torch.float16, torch.bfloat16)}


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
def test_teacher_forced_steps_match_reference(decoders, audio16, reference_ids, dt):
    res = decoders[dt].generate(audio16, PROMPT, max_new_tokens=NEW, forced_ids=reference_ids)
    torch.cuda.synchronize()
    total, same, ties = 0, 0, []
    for step, picks in enumerate(res.forced_agreement):
        for c, (ours, margin) in picks.items():
            if step >= len(reference_ids[c]):
                continue
            total += 1
            if ours == reference_ids[c][step]:
                same += 1
            else:
                ties.append((step, c, margin))
    print(f"\n{dt}: {same}/{total} steps pick the reference's token; "
          f"disagreements (step, chunk, margin): {ties}")
    near = NEAR_TIE if dt == torch.float16 else 4 * NEAR_TIE
    assert all(m < near for _, _, m in ties), ties
    # measured: every teacher-forced step agrees; allow one near tie in 32
    assert total - same <= max(1, total // 32), (same, total)


def test_free_running_first_tokens(decoders, audio16, reference_ids):
    res = decoders[torch.float16].generate(audio16, PROMPT, max_new_tokens=NEW)
    torch.cuda.synchronize()
    firsts = [ids[0] for ids in res.per_chunk_ids]
    assert firsts == [r[0] for r in reference_ids]
    for ids in res.per_chunk_ids:
        assert 1 <= len(ids) <= NEW
        assert all(i not in EOS_IDS for i in ids[:-1])


def test_decode_is_deterministic_and_chunk_independent(decoders, audio16):
    dec = decoders[torch.bfloat16]
    a = dec.generate(audio16, PROMPT, max_new_tokens=8).per_chunk_ids
    b = dec.generate(audio16, PROMPT, max_new_tokens=8).per_chunk_ids
    one = dec.generate(audio16.view(CHUNKS, 375, -1)[1:2].contiguous(), PROMPT,
                       max_new_tokens=8).per_chunk_ids
    torch.cuda.synchronize()
    assert a == b
    assert one[0][0] == a[1][0]


def test_engine_end_to_end(weights, dev):
    eng = AsrEngine(weights=weights, device=dev)
    pcm = audio_chunks_device(2, 0, 41, dev).cpu().numpy().reshape(-1)[:700000]  # 1.46 chunks
    ids = eng.transcribe_ids(pcm, PROMPT, max_new_tokens=6)
    assert len(ids) == 2 and all(1 <= len(x) <= 6 for x in ids)
    t = eng.timings
    assert t.mel_ms > 0 and t.encode_ms > 0 and t.decode_ms > 0
    # the engine's stages equal the pieces run by hand
    mel = vlasr.logmel(torch.from_numpy(
        np.concatenate([pcm, np.zeros(960000 - pcm.size, np.float32)]).reshape(2, -1)).to(dev))
    audio = eng.encoder.encode(mel)
    again = eng.decoder.generate(audio, PROMPT, max_new_tokens=6).per_chunk_ids
    assert again == ids


def test_decoder_rejects(decoders, audio16):
    dec = decoders[torch.float16]
    with pytest.raises(vlasr.VlasrInputError, match="max_seq_len"):
        dec.generate(audio16, PROMPT, max_new_tokens=1000)


def test_graph_replay_matches_eager_steps(decoders, audio16):
    dec = decoders[torch.bfloat16]
    eager = dec.generate(audio16, PROMPT, max_new_tokens=12, graphs=False).per_chunk_ids
    graphed = dec.generate(audio16, PROMPT, max_new_tokens=12, graphs=True).per_chunk_ids
    torch.cuda.synchronize()
    assert graphed == eager


def test_fused_step_matches_cublas_step(decoders, audio16, reference_ids):
    """The fused decode layers (vl_decode_linear) and the cuBLAS path give the
    same tokens (teacher forced, fp16), both agreeing with the reference."""
    dec = decoders[torch.float16]
    res = {}
    for fused in (True, False):
        dec.fused = fused
        try:
            r = dec.generate(audio16, PROMPT, max_new_tokens=NEW, forced_ids=reference_ids)
        finally:
            dec.fused = True
        res[fused] = [[i for i, _ in (p.get(c, (None, 0)) for p in r.forced_agreement)]
                      for c in range(CHUNKS)]
    torch.cuda.synchronize()
    assert res[True] == res[False]
