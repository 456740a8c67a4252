"""CPU, multi-process: the chunk sharding and the encoder-output all-gather
of the multi-GPU path, run as world_size-2 gloo process groups on 127.0.0.1.

* shard ranges tile the chunk list exactly, in order, with equal shares when
  the world size divides the count;
* gather_outputs assembles every rank's rows in global chunk order;
* a rank that dies before the collective makes the survivor's all-gather
  fail with an error within the process-group timeout instead of hanging.
"""

from __future__ import annotations

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from vlasr.pipeline import gather_outputs, host_group_bounds, shard_range


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("total,world", [(256, 1), (256, 2), (256, 4), (256, 8), (10, 3), (3, 4)])
def test_shard_ranges_tile_the_chunks(total, world):
    ranges = [shard_range(total, r, world) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == total
    for (a0, a1), (b0, b1) in zip(ranges, ranges[1:]):
        assert a1 == b0
    sizes = [b - a for a, b in ranges]
    assert max(sizes) - min(sizes) <= 1
    if total % world == 0:
        assert len(set(sizes)) == 1


def _gather_worker(rank, world, port, frames, hidden, chunks, q):
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, timeout=datetime.timedelta(seconds=30))
        c0, c1 = shard_range(chunks, rank, world)
        # each row carries (global chunk, frame) so the order can be checked
        shard = torch.empty((c1 - c0) * frames, hidden, dtype=torch.bfloat16)
        for c in range(c0, c1):
            for f in range(frames):
                shard[(c - c0) * frames + f] = c * 10 + f
        full = torch.empty(chunks * frames, hidden, dtype=torch.bfloat16)
        gather_outputs(full, shard)
        expected = torch.arange(chunks).repeat_interleave(frames) * 10 + \
            torch.arange(frames).repeat(chunks)
        ok = torch.equal(full[:, 0].float(), expected.float()) and \
            torch.equal(full[:, -1].float(), expected.float())
        dist.destroy_process_group()
        q.put((rank, ok, None))
    except Exception as exc:  # noqa: BLE001
        q.put((rank, False, repr(exc)))


def test_gather_outputs_two_ranks_global_order():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, 2, port, 5, 16, 8, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert all(ok for _, ok, _ in results), results


def _dying_worker(rank, world, port, q):
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, timeout=datetime.timedelta(seconds=5))
        if rank == 1:
            os._exit(0)  # leaves between steps, before the collective
        full = torch.empty(4, 8)
        try:
            gather_outputs(full, torch.ones(2, 8))
            q.put((rank, "completed"))
        except Exception as exc:  # noqa: BLE001
            q.put((rank, f"error: {type(exc).__name__}"))
    except Exception as exc:  # noqa: BLE001
        q.put((rank, f"setup error: {exc!r}"))


def test_dead_rank_turns_into_an_error_not_a_hang():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    rank, outcome = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert rank == 0 and outcome.startswith("error"), outcome


def test_unequal_shards_are_rejected():
    port = _free_port()
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1)
    try:
        with pytest.raises(ValueError):
            gather_outputs(torch.empty(5, 4), torch.empty(2, 4))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("chunks,groups", [(256, 8), (32, 4), (128, 8), (3, 4), (1, 1), (8, 8), (7, 3)])
def test_host_pipeline_groups_tile_the_chunks(chunks, groups):
    b = host_group_bounds(chunks, groups)
    assert b[0][0] == 0 and b[-1][1] == chunks
    assert all(x[1] == y[0] and y[1] > y[0] for x, y in zip(b, b[1:]))
    if len(b) > 2:  # half-size first and last groups
        assert b[0][1] - b[0][0] <= b[1][1] - b[1][0]
        assert b[-1][1] - b[-1][0] <= b[-2][1] - b[-2][0]


class _ContentEngine:
    """Fake engine: chunk c (filled with the value c) decodes to [c, c+1000]."""

    def transcribe_ids(self, chunks, prompt_ids, max_new_tokens=256):
        return [[int(round(float(c[0]))), int(round(float(c[0]))) + 1000] for c in chunks]


def _sharded_worker(rank, world, port, chunks, q):
    try:
        import numpy as np
        from vlasr.engine import transcribe_ids_sharded
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, timeout=datetime.timedelta(seconds=30))
        pcm = np.repeat(np.arange(chunks, dtype=np.float32)[:, None], 480000, axis=1)
        ids = transcribe_ids_sharded(_ContentEngine(), pcm, [1, 2, 3], 8)
        dist.destroy_process_group()
        q.put((rank, ids == [[c, c + 1000] for c in range(chunks)], None))
    except Exception as exc:  # noqa: BLE001
        q.put((rank, False, repr(exc)))


@pytest.mark.parametrize("chunks", [5, 2, 1])
def test_sharded_engine_returns_every_chunk_in_order(chunks):
    """Chunk sharding of the in-process engine over 2 gloo ranks: equal and
    uneven shares, and a rank without chunks."""
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_sharded_worker, args=(r, world, port, chunks, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    assert all(ok for _, ok, _ in results), results


# ---------------------------------------------------------------------------
# Copy-engine all-gather (PeerPushGather): the host side of the handle
# exchange and the copy plan, with the CUDA IPC calls replaced by a fake.
# ---------------------------------------------------------------------------

def test_push_plan_writes_own_slot_of_every_rank():
    from vlasr.pipeline import push_plan
    for world in (1, 2, 4, 8):
        for rank in range(world):
            plan = push_plan(world, rank, 1000)
            assert [j for j, _ in plan] == [rank] + [j for j in range(world) if j != rank]
            assert all(off == rank * 1000 for _, off in plan)


class _FakeIpc:
    """Handles name (rank, offset); opening one gives base 1_000_000 * (rank + 1)."""

    def __init__(self, rank):
        self.rank = rank
        self.opened, self.closed = [], []

    def export(self, ptr):
        return (f"rank{self.rank}".encode().ljust(64, b"\0"), 64 * (self.rank + 1))

    def open(self, handle):
        peer = int(handle.rstrip(b"\0")[4:])
        assert peer != self.rank
        base = 1_000_000 * (peer + 1)
        self.opened.append(base)
        return base

    def close(self, base):
        self.closed.append(base)


def _peer_worker(rank, world, port, q):
    try:
        from vlasr.pipeline import PeerPushGather
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, timeout=datetime.timedelta(seconds=30))
        full = torch.zeros(world * 4, 8)
        ipc = _FakeIpc(rank)
        g = PeerPushGather(full, 4 * 8 * 4, None, world, rank, ipc=ipc)
        dest = list(g.dest)
        g.close()
        expect = [full.data_ptr() if j == rank else 1_000_000 * (j + 1) + 64 * (j + 1)
                  for j in range(world)]
        ok = dest == expect and sorted(ipc.closed) == sorted(ipc.opened) and \
            len(ipc.opened) == world - 1 and g.opened == []
        dist.destroy_process_group()
        q.put((rank, ok, None if ok else (dest, expect)))
    except Exception as exc:  # noqa: BLE001
        q.put((rank, False, repr(exc)))


@pytest.mark.parametrize("world", [2, 3])
def test_peer_gather_maps_every_other_rank_once(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_peer_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert all(ok for _, ok, _ in results), results
