"""Multi-GPU: the chunk-sharded layer chain with its all-gather of the
encoder-norm outputs, as one process per GPU over NCCL on 127.0.0.1.

The copy-engine gather (PeerPushGather: CUDA IPC mappings, cudaMemcpyAsync
pushes, one NCCL all-reduce as the barrier) must leave in every rank's
y_all exactly what NCCL's all_gather_into_tensor assembles from the same
shards, after several steps that alternate the double-buffered outputs.
Needs two or more GPUs (skipped otherwise); the host logic runs on CPU in
test_dist_cpu.py."""

from __future__ import annotations

import datetime
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    try:
        import torch.distributed as dist

        import vlasr
        from vlasr.pipeline import ChainShape, EncoderNormChain, shard_range
        from vlasr.synth import audio_chunks_device

        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=dev)
        vlasr.load()
        chunks = 2 * world
        c0, c1 = shard_range(chunks, rank, world)
        shape = ChainShape(chunks=c1 - c0, layers=2)
        chain = EncoderNormChain(shape, dev, seed=3, world=world, rank=rank, total_chunks=chunks,
                                 gather="copy")
        pcm = audio_chunks_device(shape.chunks, c0, 0, dev)
        for _ in range(3):  # buffers 0, 1, 0
            chain.step(pcm)
        chain.finish()
        last = chain.y_bufs[1 - chain.cur]  # the buffer the last step wrote
        ref = torch.empty_like(chain.y_all)
        dist.all_gather_into_tensor(ref, last.contiguous())
        torch.cuda.synchronize()
        ok = torch.equal(chain.y_all, ref)
        chain.close()
        dist.destroy_process_group()
        q.put((rank, ok, None))
    except Exception as exc:  # noqa: BLE001
        q.put((rank, False, repr(exc)))


def test_copy_gather_matches_nccl_all_gather():
    world = min(torch.cuda.device_count(), 4)
    if world < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
    assert all(ok for _, ok, _ in results), results
