"""Chunk pipeline of the box-scale configuration: log-mel frontend, then
`layers` x (fused residual-add + LayerNorm on [frames, hidden] and exact-erf
GELU on [frames, ffn]) per 30 s chunk, optionally sharded by chunk over the
ranks of a process group with one all-gather of the encoder-norm outputs.

This is the part of the reference's encoder stage that the fused ops cover
(VideoLingo-user native/asr/src/engine.cu:1341-1578 - layer_norm, residual
add, GELU per layer - and mel_frontend.cu:209-291).  The contractions
between them (attention, fc1/fc2 GEMMs, conv frontend) are outside this
library, so each layer's inputs stand in for their outputs: the LayerNorm
residual stream is a seeded [frames, hidden] state per chunk whose delta is
the previous layer's normalised output, and the GELU input is a seeded
[frames, ffn] buffer per chunk, as the benchmark configuration prescribes.

Two entry points:
* `step()`      - device-resident inputs (HBM throughput of the ops);
* `step_host()` - host PCM in, host mel + encoder-norm outputs out, pipelined
  over chunk groups on three streams so H2D, kernels and D2H overlap.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch

from . import ops
from .synth import CHUNK_SAMPLES

FRAMES = 1500
HIDDEN = 1280
FFN = 5120
MEL_BINS = 128
MEL_FRAMES = 3000


@dataclass
class ChainShape:
    chunks: int                 # chunks processed by this rank
    layers: int = 32
    frames: int = FRAMES
    hidden: int = HIDDEN
    ffn: int = FFN

    @property
    def rows(self) -> int:
        return self.chunks * self.frames

    def bytes_per_step(self) -> dict:
        """Algorithmic HBM bytes (read every input once, write every output once)."""
        mel = self.chunks * (CHUNK_SAMPLES * 4 + MEL_BINS * MEL_FRAMES * 4)
        ln = 4 * self.rows * self.hidden * 2            # residual, delta in; residual, out
        gelu = 2 * self.rows * self.ffn * 2             # in, out
        return {"mel": mel, "add_layernorm": ln, "gelu": gelu,
                "total": mel + self.layers * (ln + gelu)}


def gather_outputs(full: torch.Tensor, shard: torch.Tensor, group=None) -> None:
    """All-gather every rank's encoder-norm rows into `full` in global chunk
    order (rank r's contiguous chunk range lands at its offset).  Requires
    equal shards, i.e. world size dividing the chunk count, as the
    benchmark's 256 chunks over 1/2/4/8 ranks do."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    if full.shape[0] != shard.shape[0] * world or full.shape[1:] != shard.shape[1:]:
        raise ValueError("gather_outputs needs equal shards: full rows = world * shard rows")
    dist.all_gather_into_tensor(full, shard.contiguous(), group=group)


def push_plan(world: int, rank: int, shard_bytes: int) -> list[tuple[int, int]]:
    """(destination rank, byte offset in its full buffer) of each copy rank
    `rank` makes per step: its shard goes to its own slot of every rank's
    full buffer, its own first."""
    order = [rank] + [j for j in range(world) if j != rank]
    return [(j, rank * shard_bytes) for j in order]


class LibIpc:
    """The C ABI's peer-memory calls (vl_ipc_export / _open / _close,
    vl_copy_async) with Python types."""

    def __init__(self):
        from . import _lib
        self._lib = _lib
        self.lib = _lib.load()

    def export(self, ptr: int) -> tuple[bytes, int]:
        import ctypes
        handle = (ctypes.c_char * self._lib.VL_IPC_HANDLE_BYTES)()
        offset = ctypes.c_uint64()
        self._lib.check(self.lib.vl_ipc_export(ctypes.c_void_p(ptr), handle, ctypes.byref(offset)),
                        "vl_ipc_export")
        return bytes(handle), int(offset.value)

    def open(self, handle: bytes) -> int:
        import ctypes
        base = ctypes.c_void_p()
        self._lib.check(self.lib.vl_ipc_open(handle, ctypes.byref(base)), "vl_ipc_open")
        return int(base.value)

    def close(self, base: int) -> None:
        self.lib.vl_ipc_close(base)

    def copy(self, dst: int, src: int, nbytes: int, stream: int) -> None:
        self._lib.check(self.lib.vl_copy_async(dst, src, nbytes, stream), "vl_copy_async")


class PeerPushGather:
    """All-gather of equal row shards with the GPUs' copy engines.

    Every rank maps every other rank's full output buffer once (CUDA IPC
    through vl_ipc_export / vl_ipc_open) and, each step, copies its own shard
    into its slot of every rank's buffer (vl_copy_async, one stream per
    destination), so no kernel and no SM takes part in the exchange.  A
    rank's copies only read its own finished shard and only write its own
    slot elsewhere, so a step needs no cross-rank ordering; `barrier()` - a
    one-element all-reduce on the caller's stream - is the point after which
    every rank's copies into this rank's buffer are complete.  `ipc`
    replaces the C ABI calls (tests)."""

    def __init__(self, full: torch.Tensor, shard_bytes: int, group, world: int, rank: int,
                 ipc=None):
        import torch.distributed as dist
        self.ipc = ipc if ipc is not None else LibIpc()
        self.full = full
        self.shard_bytes = shard_bytes
        self.group, self.world, self.rank = group, world, rank
        records = [None] * world
        dist.all_gather_object(records, self.ipc.export(full.data_ptr()), group=group)
        self.dest = [0] * world
        self.opened = []
        for j, (handle, offset) in enumerate(records):
            if j == rank:
                self.dest[j] = full.data_ptr()
                continue
            base = self.ipc.open(handle)
            self.opened.append(base)
            self.dest[j] = base + offset
        self.streams = None
        self.flag = torch.zeros(1, dtype=torch.int32, device=full.device)

    def push(self, shard: torch.Tensor, stream: torch.cuda.Stream) -> None:
        """Copy `shard` (this rank's rows, ready on `stream`) into every rank's
        full buffer; `stream` waits for all the copies."""
        if shard.numel() * shard.element_size() != self.shard_bytes or not shard.is_contiguous():
            raise ValueError("shard must be contiguous and shard_bytes long")
        if self.streams is None:
            self.streams = [torch.cuda.Stream(self.full.device) for _ in range(self.world)]
        start = torch.cuda.Event()
        start.record(stream)
        for j, off in push_plan(self.world, self.rank, self.shard_bytes):
            s = self.streams[j]
            s.wait_event(start)
            self.ipc.copy(self.dest[j] + off, shard.data_ptr(), self.shard_bytes, s.cuda_stream)
            done = torch.cuda.Event()
            done.record(s)
            stream.wait_event(done)

    def barrier(self, stream: torch.cuda.Stream) -> None:
        """Order `stream` after every rank's copies enqueued so far."""
        import torch.distributed as dist
        with torch.cuda.stream(stream):
            dist.all_reduce(self.flag, group=self.group)

    def close(self) -> None:
        """Unmap the peers' buffers, once every rank has finished its copies."""
        import torch.distributed as dist
        if self.full.is_cuda:
            torch.cuda.synchronize(self.full.device)
        dist.barrier(group=self.group)
        for base in self.opened:
            self.ipc.close(base)
        self.opened = []
        dist.barrier(group=self.group)


EDGE_MAX_CHUNKS = 4
# chunks per mel batch in vl_logmel (csrc/vl_mel.cu kBatchChunks): each batch
# is one tile launch and one normalise launch
MEL_BATCH_CHUNKS = 64


def host_group_bounds(chunks: int, groups: int) -> list[tuple[int, int]]:
    """Chunk groups of the host-buffer pipeline: `groups` equal middle groups
    plus a small first and last group (half a middle group, at most
    EDGE_MAX_CHUNKS chunks), so the upload that nothing overlaps (the first)
    and the download that nothing overlaps (the last) are short."""
    if groups <= 1 or chunks < 4:
        return [(0, chunks)]
    edge = max(1, min(EDGE_MAX_CHUNKS, chunks // (2 * groups)))
    inner = [shard_range(chunks - 2 * edge, g, groups - 1) for g in range(groups - 1)]
    bounds = [(0, edge)] + [(edge + a, edge + b) for a, b in inner if b > a]
    bounds.append((chunks - edge, chunks))
    return bounds


def shard_range(total: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous chunk range [begin, end) of `rank`; equal shares when world divides total."""
    base, extra = divmod(total, world)
    begin = rank * base + min(rank, extra)
    return begin, begin + base + (1 if rank < extra else 0)


class EncoderNormChain:
    """Resident buffers and launch sequence of one rank's shard."""

    GATHERS = ("copy", "nccl", "blocking")

    def __init__(self, shape: ChainShape, device, seed: int = 0, group=None, world: int = 1,
                 rank: int = 0, total_chunks: int | None = None, gather: str = "copy"):
        """gather (world > 1): "copy" - copy-engine pushes of each step's
        outputs into every rank's buffer, overlapped with the next step
        (PeerPushGather); "nccl" - NCCL all_gather_into_tensor on a side
        stream, overlapped; "blocking" - NCCL at the end of each step."""
        if gather not in self.GATHERS:
            raise ValueError(f"gather must be one of {self.GATHERS}")
        self.shape = shape
        self.device = torch.device(device)
        self.group = group
        self.world = world
        self.rank = rank
        self.total_chunks = total_chunks if total_chunks is not None else shape.chunks * world
        self.gather = gather
        self.overlap_gather = gather != "blocking"
        s = shape
        gen = torch.Generator(device=self.device)
        gen.manual_seed(seed * 7919 + rank)
        bf = torch.bfloat16

        def normal(shape_, mean=0.0, std=1.0):
            t = torch.empty(shape_, device=self.device, dtype=torch.float32)
            t.normal_(mean, std, generator=gen)
            return t.to(bf)

        self.gamma = normal((s.layers, s.hidden), 1.0, 0.02)
        self.beta = normal((s.layers, s.hidden), 0.0, 0.02)
        self.h = normal((s.rows, s.hidden))          # residual stream
        # LN output = next layer's delta.  Two buffers when sharded: step i's
        # outputs are all-gathered on a side stream while step i+1 computes
        # into the other buffer.
        self.y_bufs = [normal((s.rows, s.hidden))]
        if world > 1 and self.overlap_gather:
            self.y_bufs.append(normal((s.rows, s.hidden)))
        self.cur = 0
        self.g_in = normal((s.rows, s.ffn))          # FFN hidden (stand-in for fc1 output)
        self.g_out = torch.empty((s.rows, s.ffn), device=self.device, dtype=bf)
        self.mel = torch.empty((s.chunks, MEL_BINS, MEL_FRAMES), device=self.device,
                               dtype=torch.float32)
        self.mel_ws = torch.empty(ops.logmel_workspace_bytes(max(s.chunks, 1)), device=self.device,
                                  dtype=torch.uint8)
        self.y_all = None
        self.comm = None
        self.peers = None
        self.gather_done = [None, None]
        # step_host: one CUDA graph per (chunk group, output buffer, PCM buffer)
        self._group_graphs: dict[tuple[int, int, int, int], torch.cuda.CUDAGraph] = {}
        if world > 1:
            self.y_all = torch.empty((self.total_chunks * s.frames, s.hidden), device=self.device,
                                     dtype=bf)
            self.comm = torch.cuda.Stream(self.device)
            if gather == "copy":
                if self.total_chunks != s.chunks * world:
                    raise ValueError("the copy gather needs equal shards")
                self.peers = PeerPushGather(self.y_all, s.rows * s.hidden * 2, group, world, rank)

    @property
    def y(self) -> torch.Tensor:
        """The LN-output buffer of the current step."""
        return self.y_bufs[self.cur]

    # -- launch sequences ---------------------------------------------------
    def launches_per_step(self, groups: int = 1) -> int:
        """Kernels of this library launched by one step (mel: a tile and a
        normalise launch per batch of at most MEL_BATCH_CHUNKS chunks)."""
        per_group = math.ceil(self.shape.chunks / groups)
        mel = 0
        left = self.shape.chunks
        while left > 0:
            n = min(per_group, left)
            mel += 2 * math.ceil(n / MEL_BATCH_CHUNKS)
            left -= n
        return mel + 2 * self.shape.layers * groups

    def run_mel(self, pcm: torch.Tensor, c0: int = 0, c1: int | None = None) -> None:
        c1 = self.shape.chunks if c1 is None else c1
        ops.logmel(pcm[c0:c1], out=self.mel[c0:c1], workspace=self.mel_ws)

    def run_layer(self, l: int, r0: int = 0, r1: int | None = None) -> None:
        r1 = self.shape.rows if r1 is None else r1
        y = self.y[r0:r1]
        ops.add_layernorm(self.h[r0:r1], y, self.gamma[l], self.beta[l], out=y)
        ops.gelu_erf(self.g_in[r0:r1], out=self.g_out[r0:r1])

    def all_gather(self) -> None:
        """All-gather of this step's outputs, ordered on the current stream."""
        if self.y_all is None:
            return
        if self.peers is not None:
            self.peers.push(self.y, torch.cuda.current_stream(self.device))
        else:
            gather_outputs(self.y_all, self.y, self.group)

    def _begin_step(self) -> None:
        """Before writing this step's buffer: wait until its previous gather is done."""
        ev = self.gather_done[self.cur]
        if ev is not None:
            torch.cuda.current_stream(self.device).wait_event(ev)

    def _end_step(self, timer=None) -> None:
        """Start the all-gather of this step's outputs on the side stream (it
        overlaps the next step's kernels) and switch to the other buffer."""
        if self.world > 1 and not self.overlap_gather:
            if timer is not None:
                timer("all_gather", self.all_gather)
            else:
                self.all_gather()
        elif self.world > 1:
            ready = torch.cuda.Event()
            ready.record(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(self.comm):
                self.comm.wait_event(ready)
                if timer is not None:
                    timer("all_gather", self.all_gather, self.comm)
                else:
                    self.all_gather()
                done = torch.cuda.Event()
                done.record(self.comm)
            self.gather_done[self.cur] = done
            self.cur = 1 - self.cur

    def finish(self) -> None:
        """Make the current stream wait for every outstanding all-gather (with
        the copy gather: for every rank's copies into this rank's y_all).
        Collective when world > 1: every rank calls it at the same point."""
        cur = torch.cuda.current_stream(self.device)
        for ev in self.gather_done:
            if ev is not None:
                cur.wait_event(ev)
        if self.peers is not None:
            self.peers.barrier(cur)

    def close(self) -> None:
        """Release the peer mappings of the copy gather (collective)."""
        if self.peers is not None:
            self.peers.close()
            self.peers = None

    def step(self, pcm: torch.Tensor, timer=None) -> None:
        """One pass over this rank's chunks with device-resident PCM.

        `timer(name, fn[, stream])` (optional) wraps each launch, e.g. with
        CUDA events.  When sharded, the step ends by starting the all-gather
        of its outputs on a side stream; call finish() before reading y_all."""
        call = timer if timer is not None else (lambda name, fn, stream=None: fn())
        self._begin_step()
        y = self.y
        call("mel", lambda: self.run_mel(pcm))
        for l in range(self.shape.layers):
            call("add_layernorm", lambda l=l: ops.add_layernorm(
                self.h, y, self.gamma[l], self.beta[l], out=y))
            call("gelu", lambda: ops.gelu_erf(self.g_in, out=self.g_out))
        self._end_step(timer)

    # -- host-buffer path -----------------------------------------------------
    def _run_group(self, pcm_dev: torch.Tensor, c0: int, c1: int) -> None:
        """Mel + every layer of chunks [c0, c1): 2 + 2 * layers launches."""
        s = self.shape
        self.run_mel(pcm_dev, c0, c1)
        r0, r1 = c0 * s.frames, c1 * s.frames
        for l in range(s.layers):
            self.run_layer(l, r0, r1)

    def _group_graph(self, pcm_dev: torch.Tensor, c0: int, c1: int) -> torch.cuda.CUDAGraph:
        """The CUDA graph of _run_group(c0, c1) into the current output buffer,
        captured on first use.  A replay is one launch on the host where the
        group's own sequence is 66 library calls (2 + 2 x 32 layers): with
        several chunk groups per step and one process per GPU, those calls
        took as long as the GPU work itself, and the kernels waited for them."""
        key = (c0, c1, self.cur, pcm_dev.data_ptr())
        graph = self._group_graphs.get(key)
        if graph is None:
            ops.init(self.device)  # first-use set-up (tables, attributes) outside the capture
            keep = self.cur
            # both output buffers at once when they alternate, so that no
            # later step captures (a capture synchronises the device)
            for buf in range(len(self.y_bufs)):
                self.cur = buf
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    self._run_group(pcm_dev, c0, c1)
                self._group_graphs[(c0, c1, buf, pcm_dev.data_ptr())] = g
            self.cur = keep
            graph = self._group_graphs[key]
        return graph

    def release_graphs(self) -> None:
        """Drop step_host's captured group graphs."""
        self._group_graphs.clear()

    def step_host(self, pcm_host: torch.Tensor, mel_host: torch.Tensor, y_host: torch.Tensor,
                  pcm_dev: torch.Tensor, groups: int = 4, trace: list | None = None,
                  graphs: bool = True) -> None:
        """Host PCM [chunks, 480000] -> host mel [chunks,128,3000] and host
        encoder-norm outputs [chunks*frames, hidden] (pinned buffers).

        Chunk groups flow through three streams: group g+1's PCM uploads while
        group g computes and group g-1's results download.  With `graphs`
        (default), each group's computation is a CUDA graph replay, captured
        on the first call with these groups (for both output buffers when
        sharded); that call therefore synchronises the device and must not
        itself run inside a capture.  With `trace` (a list), (kind,
        start, end) CUDA event pairs are appended for every upload ("h2d"),
        group computation ("compute") and download ("d2h")."""
        s = self.shape
        bounds = host_group_bounds(s.chunks, groups)
        group_graphs = [self._group_graph(pcm_dev, c0, c1) for c0, c1 in bounds] if graphs \
            else None
        cur = torch.cuda.current_stream(self.device)
        up = torch.cuda.Stream(self.device)
        down = torch.cuda.Stream(self.device)

        def mark(stream):
            if trace is None:
                return None
            ev = torch.cuda.Event(enable_timing=True)
            ev.record(stream)
            return ev

        self._begin_step()
        uploaded = []
        up.wait_stream(cur)
        with torch.cuda.stream(up):
            for c0, c1 in bounds:
                a = mark(up)
                pcm_dev[c0:c1].copy_(pcm_host[c0:c1], non_blocking=True)
                ev = torch.cuda.Event(enable_timing=trace is not None)
                ev.record(up)
                uploaded.append(ev)
                if trace is not None:
                    trace.append(("h2d", a, ev))
        for g, ((c0, c1), ev) in enumerate(zip(bounds, uploaded)):
            cur.wait_event(ev)
            a = mark(cur)
            if group_graphs is not None:
                group_graphs[g].replay()
            else:
                self._run_group(pcm_dev, c0, c1)
            r0, r1 = c0 * s.frames, c1 * s.frames
            done = torch.cuda.Event(enable_timing=trace is not None)
            done.record(cur)
            if trace is not None:
                trace.append(("compute", a, done))
            down.wait_event(done)
            with torch.cuda.stream(down):
                a = mark(down)
                mel_host[c0:c1].copy_(self.mel[c0:c1], non_blocking=True)
                y_host[r0:r1].copy_(self.y[r0:r1], non_blocking=True)
                if trace is not None:
                    trace.append(("d2h", a, mark(down)))
        cur.wait_stream(down)
        self._end_step()

    def host_bytes_per_step(self) -> tuple[int, int]:
        s = self.shape
        h2d = s.chunks * CHUNK_SAMPLES * 4
        d2h = s.chunks * MEL_BINS * MEL_FRAMES * 4 + s.rows * s.hidden * 2
        return h2d, d2h


def seeded_pcm(chunks: int, first_chunk: int, seed: int = 0) -> np.ndarray:
    """[chunks, 480000] f32 seeded audio for global chunks first_chunk.. (config 0 recipe)."""
    from .synth import audio_chunk
    out = np.empty((chunks, CHUNK_SAMPLES), dtype=np.float32)
    for i in range(chunks):
        out[i] = audio_chunk(seed * 100003 + first_chunk + i)
    return out
