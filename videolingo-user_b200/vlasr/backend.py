"""AsrBackend over the in-process engine: `transcribe(audio_path, language)
-> Transcription`, the contract of VideoLingo-user's ASR stage
(pipeline/asr/contracts.py:6-28), with the engine subprocess of its native
backend (pipeline/asr/native.py:119-276) replaced by vlasr.engine.AsrEngine.

The flow and the error taxonomy follow the native backend: decode the file to
16 kHz mono f32 PCM, cut it into whole 30 s chunks (the tail padded with
silence, 1..128 chunks), build the shared transcription prompt once from the
first chunk, generate ids for every chunk in one batched engine call, decode
them to text, align words per spoken chunk, and return one segment per
spoken chunk with clamped word times.  Failures raise StageError.

The processor (prompt + tokenizer), the forced aligner and the language
resolver are models or libraries outside this repository; they are passed
in (or the processor is loaded from the checkpoint directory with
transformers), so the backend runs with whatever the deployment provides.
"""

from __future__ import annotations

import subprocess
import sys
import tempfile
import time
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from .synth import SAMPLE_RATE

MAX_OVERRUN = 0.5          # seconds a word or segment may run past its bound
MAX_CHUNKS = 128


class StageError(RuntimeError):
    """A pipeline stage failed (the reference's pipeline.contracts.StageError)."""


@dataclass(frozen=True)
class Word:
    text: str
    start: float
    end: float


@dataclass(frozen=True)
class TranscriptSegment:
    start: float
    end: float
    text: str
    words: tuple[Word, ...]


@dataclass(frozen=True)
class Transcription:
    language: str
    segments: tuple[TranscriptSegment, ...]


def ffmpeg_pcm(audio_path, sample_rate: int = SAMPLE_RATE) -> np.ndarray:
    """Decode any audio file to mono f32 PCM with ffmpeg (native.py:135-146)."""
    with tempfile.TemporaryDirectory(prefix="vlasr-asr-") as work:
        pcm_path = Path(work) / "audio.f32"
        try:
            run = subprocess.run(
                ["ffmpeg", "-v", "error", "-i", str(audio_path), "-ac", "1", "-ar",
                 str(sample_rate), "-f", "f32le", "-y", str(pcm_path)], capture_output=True)
        except FileNotFoundError as exc:
            raise StageError("ffmpeg is required to decode audio") from exc
        if run.returncode != 0:
            raise StageError(f"ffmpeg failed to decode audio: {run.stderr.decode()[:200]}")
        return np.fromfile(pcm_path, dtype=np.float32)


def clamp_words(timestamps, offset: float, chunk_duration: float) -> list[Word]:
    """Aligner word times (chunk-relative) -> absolute, clamped to the chunk
    [offset, offset + chunk_duration] with 1 ms minimum length, rounded to
    ms; words starting far outside the chunk are errors (the rules of the
    reference's pipeline/asr/glm.py:207-241)."""
    chunk_end = offset + chunk_duration
    words = []
    for item in timestamps:
        text = str(item.get("text", "")).strip()
        if not text:
            continue
        start = offset + float(item["start_time"])
        end = offset + float(item["end_time"])
        if start < offset - 0.05 or start > chunk_end + MAX_OVERRUN:
            raise StageError(f"forced aligner word starts outside its chunk: {start:.3f}s")
        if end < start:
            raise StageError("forced aligner returned end before start")
        if start > chunk_end:
            start, end = max(offset, chunk_end - 0.001), chunk_end
        if end == start:
            end = min(start + 0.001, chunk_end)
            if end <= start:
                start, end = max(offset, chunk_end - 0.001), chunk_end
        end = min(end, chunk_end)
        if end <= start:
            start, end = min(start, chunk_end - 0.001), chunk_end
        start, end = round(start, 3), round(end, 3)
        if end <= start:
            end = round(min(chunk_end, start + 0.001), 3)
        if end <= start:
            start = round(max(offset, end - 0.001), 3)
        if end <= start:
            raise StageError("forced aligner produced a zero-length word")
        words.append(Word(text=text, start=start, end=end))
    return words


def _default_language(configured, texts) -> str:
    if configured is not None and str(configured).strip() and str(configured).lower() != "auto":
        return str(configured).strip()
    raise StageError("cannot detect language without a language resolver; set the language")


class VlasrAsrBackend:
    """AsrBackend over AsrEngine.

    engine       an AsrEngine, or None to build one from model_dir on first use
    processor    object with apply_transcription_request([pcm]).input_ids and
                 tokenizer.decode(ids, skip_special_tokens=True); None loads
                 transformers' AutoProcessor from model_dir
    aligner      callable(arrays, texts, language) -> per-text lists of
                 {"text", "start_time", "end_time"} (chunk-relative seconds);
                 None skips word alignment: every segment spans its chunk
    language_resolver  callable(configured, texts) -> language code
    audio_loader callable(path) -> mono f32 16 kHz PCM (default ffmpeg)
    group        a torch.distributed process group: every rank runs the same
                 call; the chunks are sharded over the ranks (one GPU each)
                 and every rank returns the whole transcription
    """

    def __init__(self, model_dir=None, *, engine=None, processor=None, aligner=None,
                 language_resolver=None, audio_loader=None, chunk_seconds: float = 30.0,
                 max_new_tokens: int = 256, aligner_batch: int = 4, group=None):
        self.model_dir = Path(model_dir) if model_dir is not None else None
        self.engine = engine
        self.processor = processor
        self.aligner = aligner
        self.language_resolver = language_resolver or _default_language
        self.audio_loader = audio_loader or ffmpeg_pcm
        self.chunk_seconds = float(chunk_seconds)
        self.max_new_tokens = int(max_new_tokens)
        self.aligner_batch = int(aligner_batch)
        self.group = group      # a torch.distributed group: shard the chunks over its ranks

    def _engine(self):
        if self.engine is None:
            if self.model_dir is None or not self.model_dir.is_dir():
                raise StageError(f"ASR model dir not found: {self.model_dir}")
            from .engine import AsrEngine
            self.engine = AsrEngine(self.model_dir)
        return self.engine

    def _processor(self):
        if self.processor is None:
            if self.model_dir is None:
                raise StageError("a processor or a model_dir is required")
            from transformers import AutoProcessor
            self.processor = AutoProcessor.from_pretrained(str(self.model_dir))
        return self.processor

    def transcribe(self, audio_path, language=None) -> Transcription:
        started = time.perf_counter()
        chunk_samples = int(round(SAMPLE_RATE * self.chunk_seconds))
        pcm = np.asarray(self.audio_loader(audio_path), dtype=np.float32).reshape(-1)
        samples = pcm.size
        if samples == 0:
            raise StageError("decoded audio is empty")
        chunks = (samples + chunk_samples - 1) // chunk_samples
        if not 1 <= chunks <= MAX_CHUNKS:
            raise StageError(f"native ASR supports 1..{MAX_CHUNKS} chunks, got {chunks}")
        padded = np.zeros(chunks * chunk_samples, dtype=np.float32)
        padded[:samples] = pcm
        arrays = padded.reshape(chunks, chunk_samples)

        processor = self._processor()
        prompt_ids = list(processor.apply_transcription_request([arrays[0]]).input_ids[0])
        try:
            if self.group is not None:
                from .engine import transcribe_ids_sharded
                per_chunk = transcribe_ids_sharded(self._engine(), arrays, prompt_ids,
                                                   self.max_new_tokens, group=self.group)
            else:
                per_chunk = self._engine().transcribe_ids(arrays, prompt_ids,
                                                          max_new_tokens=self.max_new_tokens)
        except StageError:
            raise
        except Exception as exc:  # noqa: BLE001 - engine failures become stage errors
            raise StageError(f"ASR engine failed: {exc}") from exc
        if len(per_chunk) != chunks:
            raise StageError(f"ASR engine returned {len(per_chunk)} transcripts for {chunks} chunks")
        texts = [processor.tokenizer.decode(ids, skip_special_tokens=True).strip()
                 for ids in per_chunk]
        spoken = [(i, t) for i, t in enumerate(texts) if t]
        if not spoken:
            raise StageError("ASR returned no speech for the audio")
        for i, t in enumerate(texts):
            if not t:
                print(f"transcribe: no speech in chunk at {i * self.chunk_seconds:.1f}s",
                      file=sys.stderr)
        code = self.language_resolver(language, [t for _, t in spoken])

        if self.aligner is not None:
            aligned = []
            for b in range(0, len(spoken), self.aligner_batch):
                batch = spoken[b:b + self.aligner_batch]
                result = self.aligner([arrays[i] for i, _ in batch], [t for _, t in batch], code)
                if len(result) != len(batch):
                    raise StageError("alignment returned a wrong number of results")
                aligned.extend(result)
        else:
            aligned = [None] * len(spoken)
        segments = []
        for (index, text), stamps in zip(spoken, aligned):
            offset = index * self.chunk_seconds
            if stamps is None:
                end = min(offset + self.chunk_seconds, samples / SAMPLE_RATE)
                segments.append(TranscriptSegment(start=round(offset, 3), end=round(end, 3),
                                                  text=text, words=()))
                continue
            words = clamp_words(stamps, offset, self.chunk_seconds)
            if not words:
                raise StageError(f"forced aligner returned no words for chunk {index}")
            segments.append(TranscriptSegment(start=words[0].start, end=words[-1].end,
                                              text=text, words=tuple(words)))
        last_end = 0.0
        for seg in segments:
            if seg.start < last_end - 0.05:
                raise StageError("transcription segments overlap or regress")
            last_end = seg.end
        duration = samples / SAMPLE_RATE
        if last_end > duration + MAX_OVERRUN:
            raise StageError(f"transcription ends at {last_end:.3f}s, beyond audio duration "
                             f"{duration:.3f}s")
        print(f"transcribe[vlasr]: chunks={chunks} audio_seconds={duration:.1f} "
              f"segments={len(segments)} words={sum(len(s.words) for s in segments)} "
              f"elapsed={time.perf_counter() - started:.2f}s", file=sys.stderr)
        return Transcription(language=code, segments=tuple(segments))
