"""CPU: the AsrBackend mirror (vlasr.backend) with a fake engine, processor and
aligner - the flow, chunking, word clamping and error taxonomy of the
reference's native backend (pipeline/asr/native.py:119-276)."""

from __future__ import annotations

import numpy as np
import pytest

from vlasr.backend import StageError, VlasrAsrBackend, clamp_words
from vlasr.engine import pad_to_chunks

SR = 16000


class FakeTokenizer:
    def decode(self, ids, skip_special_tokens=True):
        return " ".join(f"w{i}" for i in ids if not (skip_special_tokens and i >= 59246))


class FakeProcessor:
    tokenizer = FakeTokenizer()

    def __init__(self):
        self.requests = 0

    def apply_transcription_request(self, arrays):
        self.requests += 1
        assert len(arrays) == 1 and arrays[0].shape == (30 * SR,)

        class R:
            input_ids = [[1, 2, 59260, 3]]
        return R()


class FakeEngine:
    def __init__(self, per_chunk):
        self.per_chunk = per_chunk
        self.calls = []

    def transcribe_ids(self, arrays, prompt_ids, max_new_tokens=256):
        self.calls.append((arrays.shape, list(prompt_ids), max_new_tokens))
        return self.per_chunk[:arrays.shape[0]]


def fake_aligner(arrays, texts, language):
    out = []
    for t in texts:
        words = t.split()
        out.append([{"text": w, "start_time": 1.0 + i, "end_time": 1.5 + i}
                    for i, w in enumerate(words)])
    return out


def backend(per_chunk, seconds, aligner=fake_aligner, **kw):
    pcm = np.zeros(int(seconds * SR), np.float32)
    return VlasrAsrBackend(engine=FakeEngine(per_chunk), processor=FakeProcessor(),
                           aligner=aligner, audio_loader=lambda path: pcm,
                           language_resolver=lambda c, t: c or "zh", **kw)


def test_chunks_prompt_and_segments():
    b = backend([[10, 11, 59253], [59246], [12, 59255]], 75.0)
    tr = b.transcribe("x.wav", language="en")
    assert tr.language == "en"
    shape, prompt, budget = b.engine.calls[0]
    assert shape == (3, 30 * SR) and prompt == [1, 2, 59260, 3] and budget == 256
    # chunk 1 is silent (only EOS): no segment for it
    assert [s.text for s in tr.segments] == ["w10 w11", "w12"]
    assert tr.segments[0].words[0].start == 1.0 and tr.segments[1].words[0].start == 61.0
    assert tr.segments[1].end == 61.5


def test_without_aligner_segments_span_chunks():
    tr = backend([[10], [11]], 45.0, aligner=None).transcribe("x.wav", language="zh")
    assert [(s.start, s.end) for s in tr.segments] == [(0.0, 30.0), (30.0, 45.0)]
    assert all(s.words == () for s in tr.segments)


@pytest.mark.parametrize("seconds,msg", [(0.0, "empty"), (30 * 129, "1..128")])
def test_audio_size_errors(seconds, msg):
    with pytest.raises(StageError, match=msg):
        backend([[1]] * 200, seconds).transcribe("x.wav")


def test_no_speech_is_an_error():
    with pytest.raises(StageError, match="no speech"):
        backend([[59253], [59246]], 40.0).transcribe("x.wav", language="zh")


def test_engine_failure_becomes_stage_error():
    class Broken:
        def transcribe_ids(self, *a, **k):
            raise RuntimeError("device lost")
    b = backend([], 10.0)
    b.engine = Broken()
    with pytest.raises(StageError, match="device lost"):
        b.transcribe("x.wav", language="zh")


def test_wrong_transcript_count():
    with pytest.raises(StageError, match="returned 1 transcripts for 2"):
        backend([[5]], 40.0).transcribe("x.wav", language="zh")


def test_clamp_words_rules():
    w = clamp_words([{"text": "a", "start_time": 0.0, "end_time": 0.0},
                     {"text": " ", "start_time": 1, "end_time": 2},
                     {"text": "b", "start_time": 29.9995, "end_time": 31.0},
                     {"text": "c", "start_time": 30.2, "end_time": 30.4}], 60.0, 30.0)
    assert [x.text for x in w] == ["a", "b", "c"]
    assert (w[0].start, w[0].end) == (60.0, 60.001)
    assert w[1].end == 90.0 and w[2].end == 90.0 and w[2].start < 90.0
    with pytest.raises(StageError, match="outside"):
        clamp_words([{"text": "z", "start_time": -1.0, "end_time": 0.5}], 0.0, 30.0)
    with pytest.raises(StageError, match="end before start"):
        clamp_words([{"text": "z", "start_time": 2.0, "end_time": 1.0}], 0.0, 30.0)


def test_pad_to_chunks():
    out = pad_to_chunks(np.ones(480000 + 10, np.float32))
    assert out.shape == (2, 480000) and out[1, 9] == 1 and out[1, 10] == 0


def test_collect_ids_stops_at_the_first_eos():
    from vlasr.decoder import collect_ids
    rows = [[5, 6, 59253, 59253, 59253], [7, -1, -1, -1, -1], [8, 9, 10, 11, 12], [59246, 1, 2]]
    assert collect_ids(rows) == [[5, 6, 59253], [7], [8, 9, 10, 11, 12], [59246]]
