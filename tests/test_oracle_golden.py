"""CPU: pin the oracle against the golden vectors before trusting it.

* mel: the float64 restatement and the fp32 restatement of the reference's
  own pipeline against transformers' WhisperFeatureExtractor outputs, with
  the reference's gate (max abs <= 1e-3, mean abs <= 1e-5;
  VideoLingo-user tests/test_native_asr_m0.py:174-190).
* layer ops: the C restatement against the transformers GLM-ASR modeling
  semantics (tests/golden/ops_hf.npz).
* the kernel's generated constant tables equal the oracle's fp64 tables
  rounded to f32, bit for bit.
"""

from __future__ import annotations

import re

import numpy as np
import pytest

import oracle
from conftest import GOLDEN, PKG
from helpers import normwise
from vlasr.synth import pad_chunk, tone_pcm


@pytest.fixture(scope="module")
def mel_golden():
    return np.load(GOLDEN / "mel_whisper.npz")


@pytest.fixture(scope="module")
def ops():
    return np.load(GOLDEN / "ops_hf.npz")


def _gate(produced, reference, max_abs=1e-3, mean_abs=1e-5):
    diff = np.abs(np.asarray(produced, np.float64) - np.asarray(reference, np.float64))
    assert diff.max() <= max_abs, diff.max()
    assert diff.mean() <= mean_abs, diff.mean()


def test_mel_f64_short_clip_matches_whisper(mel_golden):
    mel = oracle.logmel_f64(pad_chunk(tone_pcm(30000, seed=7)))[0]
    _gate(mel, mel_golden["short"])


def test_mel_f64_full_chunk_matches_whisper(mel_golden):
    mel = oracle.logmel_f64(tone_pcm(480000, seed=42))[0]
    _gate(mel[:, mel_golden["full_frames"]], mel_golden["full_subset"])
    assert abs(mel.max() - mel_golden["full_max"]) <= 1e-4
    assert abs(mel.mean() - mel_golden["full_mean"]) <= 1e-5


def test_mel_reference_restatement_matches_whisper(mel_golden):
    # The fp32 direct-DFT pipeline of mel_frontend.cu, restated in C.  The
    # reference reports max abs 9.5e-6 (short) / 9.1e-5 (30 s) against
    # WhisperFE (docs/agents/native-asr-m0.md:20-21,71).
    short = oracle.logmel_ref(pad_chunk(tone_pcm(30000, seed=7)))[0]
    _gate(short, mel_golden["short"], max_abs=2e-5)
    full = oracle.logmel_ref(tone_pcm(480000, seed=42))[0]
    _gate(full[:, mel_golden["full_frames"]], mel_golden["full_subset"], max_abs=2e-4)


def test_mel_restatements_agree_normwise():
    x = tone_pcm(480000, seed=42)
    assert normwise(oracle.logmel_ref(x), oracle.logmel_f64(x)) <= 1e-5


def test_layernorm_matches_hf(ops):
    _, out = oracle.add_layernorm(ops["ln_res"], ops["ln_delta"], ops["ln_gamma"], ops["ln_beta"],
                                  1e-5, "f32")
    assert normwise(out, ops["ln_out"]) <= 1e-6


def test_rmsnorm_matches_hf(ops):
    _, out = oracle.add_rmsnorm(ops["rms_res"], ops["rms_delta"], ops["rms_w"], 1e-5, "f32")
    assert normwise(out, ops["rms_out"]) <= 1e-6


def test_gelu_matches_hf(ops):
    out = oracle.gelu(ops["gelu_in"], None, "f32")
    assert normwise(out, ops["gelu_out"]) <= 1e-6


def test_swiglu_matches_hf(ops):
    out = oracle.swiglu(ops["swi_g"], ops["swi_u"], "f32")
    assert normwise(out, ops["swi_out"]) <= 1e-6


@pytest.mark.parametrize("which,head_dim,rot", [("enc", 64, 32), ("dec", 128, 64)])
def test_rope_matches_hf(ops, which, head_dim, rot):
    # transformers evaluates angle = pos * inv_freq in fp32 (error ~ pos * 2^-24
    # rad); the native reference and the oracle use fp64 angles, so agreement
    # is at the 1e-4 level for positions up to 4095.
    q, k = oracle.rope(ops[f"rope_{which}_q"], ops[f"rope_{which}_k"], ops[f"rope_{which}_pos"],
                       head_dim, rot, 10000.0, "f32")
    assert normwise(q, ops[f"rope_{which}_q_out"]) <= 2e-4
    assert normwise(k, ops[f"rope_{which}_k_out"]) <= 2e-4
    # the pass-through dims are untouched
    np.testing.assert_array_equal(q[..., rot:], ops[f"rope_{which}_q"][..., rot:])


def test_rounding_matches_torch():
    import torch
    x = np.random.default_rng(0).normal(0, 3, 100000).astype(np.float32)
    x[:4] = [np.inf, -np.inf, 0.0, -0.0]
    for name, dt in (("bf16", torch.bfloat16), ("f16", torch.float16)):
        ours = oracle.round_to(x, name)
        theirs = torch.from_numpy(x).to(dt).float().numpy()
        np.testing.assert_array_equal(ours, theirs)


def _parse_inc_floats(text: str, name: str) -> np.ndarray:
    body = re.search(name + r"\[\d+\] = \{(.*?)\};", text, re.S).group(1)
    vals = []
    for tok in body.replace("\n", " ").split(","):
        tok = tok.strip().rstrip("f")
        if tok:
            vals.append(float.fromhex(tok) if "p" in tok else float(tok))
    return np.array(vals, dtype=np.float32)


def test_kernel_mel_tables_equal_oracle_tables():
    import importlib.util
    gen_path = PKG / "csrc" / "gen_mel_tables.py"
    spec = importlib.util.spec_from_file_location("gen_mel_tables", gen_path)
    gen = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(gen)
    committed = (PKG / "csrc" / "mel_tables.inc").read_text()
    assert gen.render() == committed, "mel_tables.inc is stale: rerun gen_mel_tables.py"
    runs = (PKG / "csrc" / "mel_runs.inc").read_text()
    assert gen.render_runs() == runs, "mel_runs.inc is stale: rerun gen_mel_tables.py"
    # the unrolled runs cover every bin exactly once with the CSR taps
    assert runs.count("log10_floor(acc)") == 128 and runs.count("fmaf(") == len(gen.mel_csr()[2])
    fb = oracle.mel_filterbank_f64().astype(np.float32)  # [201, 128]
    weights = _parse_inc_floats(committed, "kMelWeights")
    lo, offsets, w = gen.mel_csr()
    dense = np.zeros_like(fb)
    for m in range(128):
        run = weights[offsets[m]:offsets[m + 1]]
        dense[lo[m]:lo[m] + len(run), m] = run
    np.testing.assert_array_equal(dense, fb)
    window = _parse_inc_floats(committed, "kWindow")
    n = np.arange(400)
    np.testing.assert_array_equal(window, (0.5 * (1 - np.cos(2 * np.pi * n / 400))).astype(np.float32))
