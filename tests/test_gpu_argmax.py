"""GPU: the decode-step tail (vl_argmax_eos) against the oracle's restatement
of the reference's argmax_mapped_kernel / argmax_rows_kernel
(native/asr/src/decoder.cu:573-621,755-782): ids bit-exact, including the
reference's tie order (smallest j mod 256, then smallest j), NaN / -inf rows,
rows with nothing above -1e30, frozen chunks, EOS, the output rows and the
row -> chunk map."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
import vlasr
from test_argmax_oracle_cpu import EOS, _rows

pytestmark = pytest.mark.gpu

DT = [(torch.bfloat16, "bf16"), (torch.float16, "f16"), (torch.float32, "f32")]


def _device_rows(rng, rows, vocab, dtype, dev, stride_pad=0):
    lg = _rows(rng, rows, vocab)
    t = torch.from_numpy(lg).to(dtype)              # storage values (ties survive rounding)
    buf = torch.full((rows, vocab + stride_pad), float("nan"), dtype=dtype)
    buf[:, :vocab] = t
    return buf.to(dev)[:, :vocab], t.float().numpy()


@pytest.mark.parametrize("dtype,name", DT, ids=[d[1] for d in DT])
@pytest.mark.parametrize("vocab", [64, 1024, 59264])
def test_plain_argmax_matches_oracle(dev, dtype, name, vocab):
    rng = np.random.default_rng(vocab + len(name))
    lg, ref_vals = _device_rows(rng, 37, vocab, dtype, dev, stride_pad=8)
    ids = vlasr.argmax_eos(lg)
    torch.cuda.synchronize()
    exp, _, _ = oracle.argmax_eos(ref_vals)
    assert ids.cpu().tolist() == exp.tolist()


@pytest.mark.parametrize("dtype,name", DT[:2], ids=[d[1] for d in DT[:2]])
def test_decode_tail_matches_oracle(dev, dtype, name):
    rng = np.random.default_rng(7)
    chunks, rows, vocab, L = 12, 9, 59264, 382
    lg, ref_vals = _device_rows(rng, rows, vocab, dtype, dev)
    ref_vals[1, :] = -3.0
    ref_vals[1, 59253] = 5.0                       # an EOS winner
    lg[1] = torch.from_numpy(ref_vals[1]).to(dtype).to(dev)
    row_chunk = np.array([3, 0, 7, 11, 5, 2, 9, 1, 8], np.int32)
    fin = np.zeros(chunks, np.uint8)
    fin[[7, 8]] = 1                                # frozen: no scan, no store
    cur = np.arange(chunks, dtype=np.int64) + 100
    out = np.full((16, chunks), -1, np.int64)
    pos = (L + rng.integers(0, 12, chunks)).astype(np.int32)
    pos[5] = L + 40                                # output row 41: outside the 16 rows
    exp_cur, exp_fin, exp_out = oracle.argmax_eos(
        ref_vals, row_chunk=row_chunk, finished=fin, current=cur, out=out, positions=pos,
        prompt_length=L, eos_ids=EOS)
    t = lambda a, dt: torch.from_numpy(np.ascontiguousarray(a)).to(dt).to(dev)  # noqa: E731
    d_fin, d_cur, d_out = t(fin, torch.bool), t(cur, torch.int64), t(out, torch.int64)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    vlasr.argmax_eos(lg, current=d_cur, finished=d_fin, row_chunk=t(row_chunk, torch.int32),
                     out=d_out, positions=t(pos, torch.int32),
                     prompt_length=torch.tensor(L, device=dev), eos_ids=EOS, status=status)
    torch.cuda.synchronize()
    assert d_cur.cpu().tolist() == exp_cur.tolist()
    assert d_fin.cpu().to(torch.uint8).tolist() == exp_fin.tolist()
    assert (d_out.cpu().numpy() == exp_out).all()
    assert int(status.item()) == vlasr.VL_STATUS_BAD_SLOT
    assert exp_fin[0] == 1 and exp_cur[0] == 59253   # row 1 -> chunk 0 finished on EOS


def test_decode_tail_in_a_graph_replays(dev):
    """Captured once, replayed with new logits and a new prompt length."""
    chunks, vocab = 4, 1024
    lg = torch.zeros(chunks, vocab, dtype=torch.bfloat16, device=dev)
    cur = torch.zeros(chunks, dtype=torch.int64, device=dev)
    fin = torch.zeros(chunks, dtype=torch.bool, device=dev)
    out = torch.full((8, chunks), -1, dtype=torch.int64, device=dev)
    pos = torch.full((chunks,), 10, dtype=torch.int32, device=dev)
    plen = torch.tensor(10, device=dev)

    def body():
        vlasr.argmax_eos(lg, current=cur, finished=fin, out=out, positions=pos,
                         prompt_length=plen, eos_ids=(7,), freeze_id=7)
        pos.add_(1)

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            body()
    torch.cuda.current_stream().wait_stream(side)
    for step, winners in enumerate([[1, 2, 3, 4], [5, 7, 5, 5], [9, 9, 9, 9]]):
        lg.zero_()
        for c, w in enumerate(winners):
            lg[c, w] = 1
        graph.replay()
    torch.cuda.synchronize()
    # output rows 1, 2, 3 (positions 10, 11, 12 with prompt length 10); chunk 1 froze at 7
    assert out[1:4].cpu().tolist() == [[1, 2, 3, 4], [5, 7, 5, 5], [9, -1, 9, 9]]
    assert cur.cpu().tolist() == [9, 7, 9, 9] and fin.cpu().tolist() == [False, True, False, False]
    del graph
