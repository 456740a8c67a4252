"""GLM-ASR text model: batched prefill and lockstep greedy decode over resident
weights, the decoder-side caller of the fused layer ops.

Computes what the reference's cross-chunk batched decode computes
(VideoLingo-user native/asr/src/decoder.cu:1372-1800, run_decode_batched):

    prefill, all chunks of the call together (the prompt ids are shared; the
    audio placeholders take the chunk's projector rows):
      h = embed(prompt, audio)                           vl_embed_gather
      28 x { y = RMSNorm1(h)                             vl_add_rmsnorm (fused with the
                                                         previous layer's residual add)
             qkv = y Wqkv^T                              one GEMM (q 2048 | k 512 | v 512)
             RoPE(q, k) at row % L                       vl_rope_inplace (rotary 128)
             cache[chunk][pos] = k, v                    vl_kv_append
             a = causal GQA attention (16 q / 4 kv heads) torch SDPA
             h += a Wo^T; y = RMSNorm2(h)                vl_add_rmsnorm
             g|u = y Wgu^T; m = silu(g) * u              one GEMM, vl_swiglu
             delta = m Wd^T }
      first id = argmax(lm_head(RMSNorm(h + delta)[last row]))
    lockstep decode, the active chunks only:
      h = embed(current id)                              vl_embed_gather (row map)
      28 x { y = RMSNorm1(h); qkv = y Wqkv^T
             a = attention of the token at its position,  vl_decode_attention (RoPE, KV
                 GQA over the chunk's cache               append and attention fused)
             ... as in prefill }
      next id = argmax(...); a chunk stops after an EOS id (59246, 59253, 59255)

Differences from the reference: every GEMM accumulates in fp32 (its default
accumulates in fp16), q/k/v and gate/up are single GEMMs, attention keeps
its scores on chip, the KV cache is not limited to 1024 positions, up to
16 chunks run each decode layer in five fused launches chained by
programmatic dependent launch, and the decode step is captured once in a
CUDA graph and replayed, with the finished flags read every 8 steps instead
of a host round trip and a re-compaction per step.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import ops
from ._lib import VlasrInputError

EOS_IDS = (59246, 59253, 59255)
AUDIO_TOKEN_ID = 59260
AUDIO_TOKENS_PER_CHUNK = 375
# Decode steps of up to this many chunks run the fused layers through
# vl_decode_linear (its default mma.sync kernel); larger batches run cuBLAS
# GEMMs, which measured faster per launch than either kernel of
# vl_decode_linear from 17 rows up.
FUSED_MAX_ROWS = 16


@dataclass(frozen=True)
class DecoderShape:
    hidden: int
    heads: int
    kv_heads: int
    head_dim: int
    ffn: int
    layers: int
    vocab: int
    rope_base: float = 10000.0
    eps: float = 1e-5


@dataclass
class DecodeResult:
    per_chunk_ids: list            # generated ids per chunk, through the first EOS
    steps: int                     # decode steps executed (lockstep rounds incl. the first id)
    forced_agreement: list | None = None   # teacher forcing: (argmax, margin) per step and chunk


class TextDecoder:
    """Resident text-model weights in one compute dtype and the prefill /
    decode launch sequences.  `weights` maps the official names
    (language_model.*) to device tensors."""

    def __init__(self, weights: dict, *, heads: int = 16, kv_heads: int = 4,
                 dtype=torch.bfloat16, max_seq_len: int = 1024,
                 audio_token_id: int = AUDIO_TOKEN_ID, eos_ids=EOS_IDS):
        if dtype not in (torch.bfloat16, torch.float16):
            raise VlasrInputError("TextDecoder computes in bf16 or fp16")
        emb = weights["language_model.model.embed_tokens.weight"]
        if emb.device.type != "cuda":
            raise VlasrInputError("TextDecoder weights must be CUDA tensors")
        vocab, hidden = emb.shape
        layers = 0
        while f"language_model.model.layers.{layers}.mlp.down_proj.weight" in weights:
            layers += 1
        ffn = weights["language_model.model.layers.0.mlp.gate_proj.weight"].shape[0]
        self.shape = DecoderShape(hidden=hidden, heads=heads, kv_heads=kv_heads,
                                  head_dim=hidden // heads, ffn=ffn, layers=layers, vocab=vocab)
        self.dtype = dtype
        self.device = emb.device
        self.max_seq_len = int(max_seq_len)
        self.audio_token_id = int(audio_token_id)
        self.eos_ids = tuple(int(e) for e in eos_ids)

        def w(name):
            t = weights[name].to(device=self.device, dtype=dtype).contiguous()
            # the fused projections stage vectors with 16-byte copies
            return t if t.data_ptr() % 16 == 0 else t.clone()

        self.embed = w("language_model.model.embed_tokens.weight")
        self.lm_head_t = w("language_model.lm_head.weight").t()
        self.norm_w = w("language_model.model.norm.weight")
        self.layer_w = []
        for l in range(layers):
            p = f"language_model.model.layers.{l}."
            self.layer_w.append({
                "ln1": w(p + "input_layernorm.weight"),
                "qkv_t": torch.cat([w(p + f"self_attn.{n}_proj.weight") for n in "qkv"], 0).t(),
                "o_t": w(p + "self_attn.o_proj.weight").t(),
                "ln2": w(p + "post_attention_layernorm.weight"),
                "gu_t": torch.cat([w(p + "mlp.gate_proj.weight"),
                                   w(p + "mlp.up_proj.weight")], 0).t(),
                "down_t": w(p + "mlp.down_proj.weight").t(),
            })
        self.eos = torch.tensor(self.eos_ids, device=self.device, dtype=torch.int64)
        self._states: dict = {}
        self.fused = True                # decode steps through vl_decode_linear (<= 64 chunks)
        self.last_timings = (0.0, 0.0)   # (prefill ms, decode-steps ms) of the last graphed call

    # ------------------------------------------------------------------
    def _mlp(self, lw: dict, h: torch.Tensor, o: torch.Tensor) -> torch.Tensor:
        """h += o; y = RMSNorm2(h); return down(silu(gate(y)) * up(y))."""
        s = self.shape
        y = ops.add_rmsnorm(h, o, lw["ln2"], eps=s.eps)
        gu = y @ lw["gu_t"]
        m = ops.swiglu(gu[:, :s.ffn], gu[:, s.ffn:])
        return m @ lw["down_t"]

    def _logits(self, h: torch.Tensor, delta: torch.Tensor | None) -> torch.Tensor:
        """Final RMSNorm of h + delta and the lm_head: [rows, vocab] in the
        compute dtype."""
        y = ops.add_rmsnorm(h, delta, self.norm_w, eps=self.shape.eps)
        return y @ self.lm_head_t

    def _argmax(self, h: torch.Tensor, delta: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """(ids, float32 logits); the ids in the reference's tie order."""
        logits = self._logits(h, delta)
        return ops.argmax_eos(logits), logits.float()

    def prefill(self, audio: torch.Tensor, prompt: torch.Tensor, k_cache, v_cache,
                chunk_slots: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """Run the prompt of every chunk; fill the caches; -> (first ids, logits)."""
        s = self.shape
        chunks, L = audio.shape[0], prompt.numel()
        h = ops.embed_gather(prompt, self.embed, audio=audio, audio_token_id=self.audio_token_id,
                             shared_ids=True, batch=chunks).view(chunks * L, s.hidden)
        qw, kw = s.heads * s.head_dim, s.kv_heads * s.head_dim
        pos_slots = (chunk_slots.view(chunks, 1)
                     + torch.arange(L, device=self.device).view(1, L)).reshape(-1)
        delta = None
        for l, lw in enumerate(self.layer_w):
            y = ops.add_rmsnorm(h, delta, lw["ln1"], eps=s.eps)
            qkv = y @ lw["qkv_t"]
            q, k, v = qkv[:, :qw], qkv[:, qw:qw + kw], qkv[:, qw + kw:]
            ops.rope_(q, k, head_dim=s.head_dim, rotary_dim=s.head_dim, base=s.rope_base,
                      seq_len=L)
            ops.kv_append(k, v, k_cache[l], v_cache[l], pos_slots)
            qh = q.view(chunks, L, s.heads, s.head_dim).transpose(1, 2)
            kh = k.view(chunks, L, s.kv_heads, s.head_dim).transpose(1, 2)
            vh = v.view(chunks, L, s.kv_heads, s.head_dim).transpose(1, 2)
            a = F.scaled_dot_product_attention(qh, kh, vh, is_causal=True, enable_gqa=True)
            a = a.transpose(1, 2).reshape(chunks * L, qw)
            delta = self._mlp(lw, h, a @ lw["o_t"])
        last = torch.arange(chunks, device=self.device) * L + (L - 1)
        return self._argmax(h[last].contiguous(), delta[last].contiguous())

    def step(self, ids: torch.Tensor, active: torch.Tensor, positions: torch.Tensor,
             k_cache, v_cache, chunk_slots: torch.Tensor, workspace: torch.Tensor):
        """One lockstep decode step -> (next ids, float32 logits) of the
        active rows (see step_logits)."""
        logits = self.step_logits(ids, active, positions, k_cache, v_cache, chunk_slots,
                                  workspace)
        return ops.argmax_eos(logits), logits.float()

    def step_logits(self, ids: torch.Tensor, active: torch.Tensor, positions: torch.Tensor,
                    k_cache, v_cache, chunk_slots: torch.Tensor,
                    workspace: torch.Tensor) -> torch.Tensor:
        """One lockstep decode step for the active chunks: ids [chunks] (int64)
        are the current tokens, positions [chunks] (int32) their positions;
        returns the logits of the active rows in the compute dtype.

        Up to FUSED_MAX_ROWS active chunks run the fused path: per layer
        vl_decode_linear (RMSNorm prologue + q|k|v), vl_decode_attention,
        vl_decode_linear (o, residual epilogue), vl_decode_linear (RMSNorm
        prologue + gate|up + SwiGLU epilogue), vl_decode_linear (down, residual
        epilogue) - five launches; more chunks run cuBLAS GEMMs between the
        standalone ops."""
        s = self.shape
        qw, kw = s.heads * s.head_dim, s.kv_heads * s.head_dim
        h = ops.embed_gather(ids.view(-1, 1), self.embed, row_map=active).view(-1, s.hidden)
        pos = positions[active.long()].contiguous()
        start = chunk_slots[active.long()].contiguous()
        rows = h.shape[0]
        if self.fused and rows <= FUSED_MAX_ROWS:
            return self._step_fused(h, pos, start, k_cache, v_cache, workspace)
        delta = None
        for l, lw in enumerate(self.layer_w):
            y = ops.add_rmsnorm(h, delta, lw["ln1"], eps=s.eps)
            qkv = y @ lw["qkv_t"]
            a = ops.decode_attention(qkv[:, :qw], k_cache[l], v_cache[l], pos, start,
                                     n_kv_heads=s.kv_heads, head_dim=s.head_dim,
                                     max_seq_len=self.max_seq_len, k=qkv[:, qw:qw + kw],
                                     v=qkv[:, qw + kw:], rotary_dim=s.head_dim,
                                     rope_base=s.rope_base, workspace=workspace)
            delta = self._mlp(lw, h, a @ lw["o_t"])
        return self._logits(h, delta)

    def _state(self, chunks: int) -> dict:
        """Per chunk count: KV caches, decode workspace and the step buffers a
        captured graph points at (kept for the next call of the same size)."""
        st = self._states.get(chunks)
        if st is not None:
            return st
        self._states.clear()        # one size at a time: free the previous caches first
        s, dev = self.shape, self.device
        kw = s.kv_heads * s.head_dim
        slots = chunks * self.max_seq_len
        st = {
            "k_cache": [torch.empty(slots, kw, dtype=self.dtype, device=dev)
                        for _ in range(s.layers)],
            "v_cache": [torch.empty(slots, kw, dtype=self.dtype, device=dev)
                        for _ in range(s.layers)],
            "chunk_slots": torch.arange(chunks, device=dev, dtype=torch.int64) * self.max_seq_len,
            "ws": torch.zeros(ops.decode_attention_workspace_bytes(
                chunks, s.heads, s.kv_heads, s.head_dim, self.max_seq_len),
                dtype=torch.uint8, device=dev),
            "out": torch.full((self.max_seq_len, chunks), -1, dtype=torch.int64, device=dev),
            "cur": torch.zeros(chunks, dtype=torch.int64, device=dev),
            "fin": torch.zeros(chunks, dtype=torch.bool, device=dev),
            "pos": torch.zeros(chunks, dtype=torch.int32, device=dev),
            "prompt_len": torch.zeros((), dtype=torch.int64, device=dev),
            "rows": torch.arange(chunks, device=dev, dtype=torch.int32),
            "graph": None,
        }
        self._states[chunks] = st
        return st

    def _decode_body(self, st: dict) -> None:
        """One lockstep step over every chunk of `st` (device state only):
        the layers, then one vl_argmax_eos launch for the reference's tail
        (argmax_mapped_kernel: freeze finished chunks, store the id at row
        position - prompt length + 1, finish on EOS, update the current ids)
        and the position advance."""
        logits = self.step_logits(st["cur"], st["rows"], st["pos"], st["k_cache"],
                                  st["v_cache"], st["chunk_slots"], st["ws"])
        ops.argmax_eos(logits, current=st["cur"], finished=st["fin"], out=st["out"],
                       positions=st["pos"], prompt_length=st["prompt_len"],
                       eos_ids=self.eos_ids, freeze_id=self.eos_ids[1])
        st["pos"].add_(1)

    def _generate_graphed(self, st: dict, first: torch.Tensor, L: int,
                          max_new_tokens: int) -> torch.Tensor:
        """Lockstep decode with the step captured in a CUDA graph (once per
        chunk count; later calls replay it).

        Every chunk stays in the batch; a finished chunk emits 59253 (the
        reference's argmax_mapped_kernel freeze) into the current ids and
        stores nothing.  Without a graph yet, step 1 runs eagerly (it also
        warms the libraries up) before the capture; the finished flags are
        read every 8 steps."""
        out = st["out"]
        out.fill_(-1)
        out[0] = first
        st["cur"].copy_(first)
        torch.isin(first, self.eos, out=st["fin"])
        st["pos"].fill_(L)
        st["prompt_len"].fill_(L)
        if max_new_tokens <= 1:
            return out[:max_new_tokens]
        dev = self.device
        step = 1
        if st["graph"] is None:
            side = torch.cuda.Stream(dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side):
                self._decode_body(st)                   # step 1, eagerly
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=side):
                    self._decode_body(st)
            torch.cuda.current_stream(dev).wait_stream(side)
            st["graph"] = graph
            step = 2
        for step in range(step, max_new_tokens):
            if step % 8 == 0 and bool(st["fin"].all()):
                break
            st["graph"].replay()
        return out[:max_new_tokens]

    def replay_step(self, chunks: int, times: int = 1) -> None:
        """Replay the captured decode step of `chunks` chunks `times` more
        times, continuing from the state the last generate() left (for timing
        the step alone).  The positions (and with them the id rows) must stay
        inside the KV caches."""
        st = self._states.get(chunks)
        if st is None or st["graph"] is None:
            raise VlasrInputError(f"no captured decode step for {chunks} chunks: run generate()")
        last = int(st["pos"].max().item()) + times
        if last >= self.max_seq_len:
            raise VlasrInputError(f"{times} more steps would pass max_seq_len {self.max_seq_len}")
        for _ in range(times):
            st["graph"].replay()

    def _step_fused(self, h: torch.Tensor, pos: torch.Tensor, start: torch.Tensor, k_cache,
                    v_cache, workspace: torch.Tensor):
        """The five launches per layer run as programmatic dependents of the
        launch before them (each streams weights, or cache rows of earlier
        steps, while that one finishes): no launch of the step writes a
        weight, the positions or slot starts, or a cache row before the
        positions."""
        s = self.shape
        rows = h.shape[0]
        qw, kw = s.heads * s.head_dim, s.kv_heads * s.head_dim
        parts = s.hidden // 16
        ssq_a = torch.empty(parts, rows, dtype=torch.float32, device=self.device)
        ssq_b = torch.empty(parts, rows, dtype=torch.float32, device=self.device)
        for l, lw in enumerate(self.layer_w):
            if l == 0:      # the embedding rows have no partial sums: normalise them first
                x = ops.add_rmsnorm(h, None, lw["ln1"], eps=s.eps)
                qkv = ops.decode_linear(x, lw["qkv_t"].t(), pdl=True)
            else:
                qkv = ops.decode_linear(h, lw["qkv_t"].t(), norm_weight=lw["ln1"], ssq_in=ssq_a,
                                        eps=s.eps, pdl=True)
            a = ops.decode_attention(qkv[:, :qw], k_cache[l], v_cache[l], pos, start,
                                     n_kv_heads=s.kv_heads, head_dim=s.head_dim,
                                     max_seq_len=self.max_seq_len, k=qkv[:, qw:qw + kw],
                                     v=qkv[:, qw + kw:], rotary_dim=s.head_dim,
                                     rope_base=s.rope_base, workspace=workspace, pdl=True)
            ops.decode_linear(a, lw["o_t"].t(), epilogue="residual", out=h, ssq_out=ssq_b,
                              pdl=True)
            m = ops.decode_linear(h, lw["gu_t"].t(), norm_weight=lw["ln2"], ssq_in=ssq_b,
                                  eps=s.eps, epilogue="swiglu", pdl=True)
            ops.decode_linear(m, lw["down_t"].t(), epilogue="residual", out=h,
                              ssq_out=ssq_a if l + 1 < s.layers else None, pdl=True)
        # final norm + lm_head: 3704 column tiles that would each re-read the
        # rows; one norm launch and the cuBLAS GEMM stream the 243 MB faster
        return self._logits(h, None)

    def generate(self, audio: torch.Tensor, prompt_ids, max_new_tokens: int = 256,
                 forced_ids: list | None = None, graphs: bool = True) -> DecodeResult:
        """audio [chunks*375, hidden] (or [chunks, 375, hidden]) projector rows;
        prompt_ids: the shared prompt (int64).  Greedy decode of up to
        max_new_tokens ids per chunk (the first from the prefill).

        forced_ids (tests): per-chunk id lists fed back instead of the argmax
        (teacher forcing); the result then records this decoder's argmax and
        its top-1/top-2 logit margin at every step."""
        s = self.shape
        prompt = torch.as_tensor(prompt_ids, dtype=torch.int64).to(self.device).contiguous()
        L = prompt.numel()
        if audio.dim() == 2:
            audio = audio.view(-1, AUDIO_TOKENS_PER_CHUNK, s.hidden)
        audio = audio.to(self.dtype).contiguous()
        chunks = audio.shape[0]
        if L + max_new_tokens > self.max_seq_len:
            raise VlasrInputError("prompt plus budget exceeds the decoder's max_seq_len")
        if chunks < 1:
            raise VlasrInputError("at least one chunk is required")
        st = self._state(chunks)
        k_cache, v_cache = st["k_cache"], st["v_cache"]
        chunk_slots, ws = st["chunk_slots"], st["ws"]
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        ev[0].record()
        first, logits = self.prefill(audio, prompt, k_cache, v_cache, chunk_slots)
        ev[1].record()
        if graphs and forced_ids is None:
            out = self._generate_graphed(st, first, L, max_new_tokens)
            ev[2].record()
            result = DecodeResult(per_chunk_ids=self._collect(out, chunks),
                                  steps=int((out >= 0).any(1).sum()))
            self.last_timings = (ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2]))
            return result
        out = torch.full((max_new_tokens, chunks), -1, dtype=torch.int64, device=self.device)
        agreement = [] if forced_ids is not None else None

        def record(step_ids, lg, rows):
            if agreement is None:
                return
            top2 = lg.topk(2, dim=-1)
            margin = (top2.values[:, 0] - top2.values[:, 1]).tolist()
            agreement.append({int(c): (int(i), float(m))
                              for c, i, m in zip(rows.tolist(), step_ids.tolist(), margin)})

        all_rows = torch.arange(chunks, device=self.device, dtype=torch.int32)
        record(first, logits, all_rows)
        current = first.clone()
        if forced_ids is not None:
            current = torch.tensor([f[0] for f in forced_ids], device=self.device)
        out[0] = current
        finished = torch.isin(current, self.eos)
        positions = torch.full((chunks,), L, dtype=torch.int32, device=self.device)
        steps = 1
        for step in range(1, max_new_tokens):
            fin = finished.tolist()
            if forced_ids is not None:
                fin = [len(forced_ids[c]) <= step for c in range(chunks)]
            act = [c for c in range(chunks) if not fin[c]]
            if not act:
                break
            active = torch.tensor(act, device=self.device, dtype=torch.int32)
            nxt, lg = self.step(current, active, positions, k_cache, v_cache, chunk_slots, ws)
            record(nxt, lg, active)
            rows = active.long()
            if forced_ids is not None:
                nxt = torch.tensor([forced_ids[c][step] for c in act], device=self.device)
            current[rows] = nxt
            out[step, rows] = nxt
            finished[rows] = torch.isin(nxt, self.eos)
            positions[rows] += 1
            steps += 1
        return DecodeResult(per_chunk_ids=self._collect(out, chunks), steps=steps,
                            forced_agreement=agreement)

    def _collect(self, out: torch.Tensor, chunks: int) -> list[list[int]]:
        return collect_ids(out.t().tolist()[:chunks], self.eos_ids)


def collect_ids(rows_per_chunk, eos_ids=EOS_IDS) -> list[list[int]]:
    """Generated-id rows per chunk (-1 = not generated) -> the ids through
    the first EOS, as the reference collects them (decoder.cu:1783-1790)."""
    eos = set(int(e) for e in eos_ids)
    per_chunk = []
    for row in rows_per_chunk:
        seq = []
        for i in row:
            if i < 0:
                break
            seq.append(int(i))
            if i in eos:
                break
        per_chunk.append(seq)
    return per_chunk
