"""CPU: the oracle of the decode-step tail (oracle.argmax_eos, the literal
256-thread loops of the reference's argmax_mapped_kernel / argmax_rows_kernel,
native/asr/src/decoder.cu:573-621,755-782) against an independent statement
of the order they produce: the largest value above -1e30, ties to the
smallest j mod 256 and then the smallest j; plus the freeze / EOS / output-row
bookkeeping."""

from __future__ import annotations

import numpy as np
import pytest

import oracle

EOS = (59246, 59253, 59255)


def rule(row: np.ndarray, empty: int) -> int:
    v = np.where(row > np.float32(-1e30), row, -np.inf)   # NaN compares false
    m = v.max()
    if m == -np.inf:
        return empty
    idx = np.flatnonzero(v == m)
    return int(idx[np.lexsort((idx, idx % 256))[0]])


def _rows(rng, rows, vocab):
    lg = rng.normal(0, 1, (rows, vocab)).astype(np.float32)
    lg = np.round(lg * 4) / 4                       # coarse values: many exact ties
    for r in range(rows):
        kind = r % 6
        m = lg[r].max() + 1
        if kind == 1:                               # the max at several j, various j mod 256
            lg[r, rng.choice(vocab, 5, replace=False)] = m
        elif kind == 2:                             # NaN and -inf never win
            lg[r, rng.choice(vocab, 7, replace=False)] = np.nan
            lg[r, rng.choice(vocab, 3, replace=False)] = -np.inf
        elif kind == 3:                             # nothing above -1e30
            lg[r] = -1e30
            lg[r, 5] = -np.inf
        elif kind == 4:                             # +inf wins; ties among infinities
            lg[r, [300 % vocab, 44 % vocab, 1000 % vocab]] = np.inf
    return lg


@pytest.mark.parametrize("vocab", [64, 1024, 59264])
def test_oracle_matches_the_tie_rule(vocab):
    rng = np.random.default_rng(vocab)
    lg = _rows(rng, 24, vocab)
    ids, _, _ = oracle.argmax_eos(lg)
    assert ids.tolist() == [rule(r, 0) for r in lg]
    ids, fin, _ = oracle.argmax_eos(lg, finished=np.zeros(24, np.uint8), current=np.zeros(24),
                                    eos_ids=EOS)
    assert ids.tolist() == [rule(r, 59253) for r in lg]


def test_known_ties():
    lg = np.full((3, 1024), -5, np.float32)
    lg[0, [45, 300]] = 7          # 300 % 256 = 44 < 45
    lg[1, [255, 511]] = 7         # same thread: the smaller j
    lg[2, [256, 1]] = 7           # thread 0 (j = 256) before thread 1
    assert oracle.argmax_eos(lg)[0].tolist() == [300, 255, 256]


def test_freeze_eos_and_output_rows():
    vocab, chunks = 59264, 4
    lg = np.zeros((3, vocab), np.float32)
    lg[0, 59255] = 9              # row 0 -> chunk 2: EOS, finishes it
    lg[1, 17] = 9                 # row 1 -> chunk 0: a word
    lg[2, 99] = 9                 # row 2 -> chunk 3: already finished, frozen
    fin = np.array([0, 0, 0, 1], np.uint8)
    cur = np.array([5, 6, 7, 8], np.int64)
    out = np.full((8, chunks), -1, np.int64)
    pos = np.array([3, 0, 11, 12], np.int32)       # per chunk
    ids, fin2, out2 = oracle.argmax_eos(lg, row_chunk=[2, 0, 3], finished=fin, current=cur,
                                        out=out, positions=pos, prompt_length=10, eos_ids=EOS)
    assert ids.tolist() == [17, 6, 59255, 59253]    # chunk 1 has no row: unchanged
    assert fin2.tolist() == [0, 0, 1, 1]
    # chunk 2 at position 11: row 11 - 10 + 1 = 2; chunk 0 at position 3: row -6, not stored;
    # chunk 3 is frozen: nothing stored
    expect = np.full((8, chunks), -1, np.int64)
    expect[2, 2] = 59255
    assert (out2 == expect).all()
