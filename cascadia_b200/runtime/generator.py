"""Batched prefill + decode for one model stage, with CUDA-graph decode.

``DecodeGraph`` captures one whole decode step of a stage (embedding, all
layers, final norm, LM head, argmax) for a fixed batch size and block-table
width.  Per step the host writes positions, KV slots, sequence lengths and the
last tokens into one pinned int32 staging buffer, issues a single
host-to-device copy, replays the graph and reads back the int32 next tokens.
This replaces the reference's per-token synchronous OpenVINO infer calls
(crates/cascadia-engine-openvino/src/runtime.rs:1666, :2602-2775).
"""
from __future__ import annotations

from typing import Dict, List, Optional, Sequence

import numpy as np
import torch

from .. import ops
from ..models.llama import Batch, build_batch
from .kv_cache import BLOCK_SIZE


class DecodeGraph:
    """A captured decode step for `batch` sequences and table width `width`."""

    def __init__(self, model, batch: int, width: int, use_graph: bool = True,
                 num_splits: Optional[int] = None):
        self.model = model
        self.B = batch
        self.W = width
        dev = model.device
        self.dev = dev
        # Layout of the staging row: ids | positions | slots | seq_lens | table
        self.n_int = 4 * batch + batch * width
        pin = torch.device(dev).type == "cuda"
        self.host = torch.zeros(self.n_int, dtype=torch.int32, pin_memory=pin)
        self.dev_in = torch.zeros(self.n_int, dtype=torch.int32, device=dev)
        b = batch
        self.ids = self.dev_in[0:b]
        self.positions = self.dev_in[b:2 * b]
        self.slots = self.dev_in[2 * b:3 * b]
        self.seq_lens = self.dev_in[3 * b:4 * b]
        self.table = self.dev_in[4 * b:].view(b, width)
        self.out_host = torch.zeros(batch, dtype=torch.int32, pin_memory=pin)
        self.hidden = torch.zeros(batch, model.cfg.hidden_size, dtype=torch.bfloat16, device=dev)
        # Pipeline stages after the first receive their input rows here; the
        # step copies them into `hidden` (the layers update it in place), so
        # replaying or re-running a step is idempotent.
        self.hidden_in = None if model.has_embed else torch.zeros(
            batch, model.payload_in_width, dtype=torch.bfloat16, device=dev)
        self.payload_out = None  # what a non-last stage sends on
        if num_splits is None:
            num_splits, bps = ops.decode_split_plan(batch, model.hkv, width)
        else:
            bps = max(1, -(-width // num_splits))
        self.num_splits, self.bps = num_splits, bps
        g = model.hq // model.hkv
        n = batch * model.hkv * num_splits * g
        self.part_o = torch.empty(max(1, n * model.d), dtype=torch.float32, device=dev)
        self.part_ml = torch.empty(max(1, n * 2), dtype=torch.float32, device=dev)
        self.batch_view = Batch(seq_ids=[f"g{i}" for i in range(b)], q_lens=[1] * b,
                                ctx_lens=[0] * b, positions=self.positions, slots=self.slots,
                                block_tables=self.table, seq_lens=self.seq_lens, is_decode=True,
                                num_splits=num_splits, blocks_per_split=bps, part_o=self.part_o,
                                part_ml=self.part_ml)
        self.next_ids = None
        self.logits = None
        self.graph = None
        self.launches = 0
        self.use_graph = use_graph and dev.type == "cuda"

    def _step(self):
        """Embedding (first stage), this stage's layers, LM head + argmax (last
        stage).  A middle or last pipeline stage finds its input rows in
        ``self.hidden_in`` (received before the replay)."""
        m = self.model
        if m.has_embed:
            m.embed_tokens(self.ids, out=self.hidden)
        else:
            m.unpack_payload(self.hidden_in, self.batch_view, out=self.hidden)
        m.forward(self.batch_view, self.hidden)
        if not m.has_head:
            self.payload_out = m.pack_payload(self.hidden, self.batch_view)
        if m.has_head:
            self.logits = m.head(self.hidden)
            self.next_ids = m.greedy(self.logits)
        return self.next_ids

    def capture(self, warmup: int = 2):
        """Capture the step into a CUDA graph (inputs must hold valid data)."""
        if not self.use_graph:
            return
        # Models with recurrent state (linear attention) advance it on every
        # step: keep the batch's state as it was before the warm-up steps.
        m = self.model
        saved = m.save_state(self.batch_view) if hasattr(m, "save_state") else None
        s = torch.cuda.Stream(device=self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(s):
            for _ in range(warmup):
                self._step()
        torch.cuda.current_stream(self.dev).wait_stream(s)
        torch.cuda.synchronize(self.dev)
        if saved is not None:
            m.restore_state(saved)
            torch.cuda.synchronize(self.dev)
        self.graph = torch.cuda.CUDAGraph()
        ops.LAUNCHES.start()
        with torch.cuda.graph(self.graph, stream=s):
            self._step()
        self.launches = ops.LAUNCHES.stop()
        torch.cuda.synchronize(self.dev)

    def fill(self, ids, positions, slots, seq_lens, table: np.ndarray):
        h = self.host.numpy()
        b = self.B
        h[0:b] = ids
        h[b:2 * b] = positions
        h[2 * b:3 * b] = slots
        h[3 * b:4 * b] = seq_lens
        h[4 * b:] = table.reshape(-1)

    def upload(self):
        self.dev_in.copy_(self.host, non_blocking=True)

    def run(self) -> torch.Tensor:
        if self.graph is not None:
            self.graph.replay()
            return self.next_ids
        return self._step()

    def download(self) -> torch.Tensor:
        self.out_host.copy_(self.next_ids, non_blocking=True)
        return self.out_host


class BatchGenerator:
    """Greedy batch generation over a single-stage model (used by tests, the
    bench and the engine's single-GPU path)."""

    def __init__(self, model, use_graph: bool = True):
        self.model = model
        self.use_graph = use_graph
        self.graphs: Dict[tuple, DecodeGraph] = {}
        self.last_hidden: Optional[torch.Tensor] = None

    def prefill(self, seq_ids: Sequence[str], prompts: Sequence[Sequence[int]],
                start: Optional[Sequence[int]] = None) -> torch.Tensor:
        m = self.model
        start = start or [0] * len(seq_ids)
        for sid in seq_ids:
            if sid not in m.kv.seqs:
                m.kv.add_sequence(sid)
        q_lens = [len(p) for p in prompts]
        batch = build_batch(m, seq_ids, q_lens, start, decode=False)
        ids = torch.tensor([t for p in prompts for t in p], dtype=torch.int32).to(m.device)
        hidden = m.embed_tokens(ids)
        m.forward(batch, hidden)
        self.last_hidden = hidden  # pre-norm rows of every prompt token (MTP drafting)
        last = torch.tensor(batch.last_rows, dtype=torch.long, device=m.device)
        logits = m.head(hidden.index_select(0, last).contiguous())
        return m.greedy(logits)

    def decode_graph(self, seq_ids: Sequence[str], width: int) -> DecodeGraph:
        key = (len(seq_ids), width)
        g = self.graphs.get(key)
        if g is None:
            g = DecodeGraph(self.model, len(seq_ids), width, self.use_graph)
            self.graphs[key] = g
        return g

    def stage_decode_inputs(self, g: DecodeGraph, seq_ids, last_tokens):
        kv = self.model.kv
        b = len(seq_ids)
        pos = np.empty(b, dtype=np.int32)
        slots = np.empty(b, dtype=np.int32)
        lens = np.empty(b, dtype=np.int32)
        table = np.zeros((b, g.W), dtype=np.int32)
        for i, sid in enumerate(seq_ids):
            s = kv.seqs[sid]
            p = s.length
            kv.reserve(sid, p + 1)
            s.length = p + 1
            pos[i] = p
            slots[i] = s.blocks[p // BLOCK_SIZE] * BLOCK_SIZE + p % BLOCK_SIZE
            lens[i] = p + 1
            kv.slide(sid, self.model.cfg, p)
            table[i, :len(s.blocks)] = np.maximum(s.blocks, 0)
        g.fill(np.asarray(last_tokens, dtype=np.int32), pos, slots, lens, table)

    def decode(self, seq_ids: Sequence[str], last_tokens, width: int) -> torch.Tensor:
        m = self.model
        if m.device.type != "cuda":
            starts = [m.kv.seqs[s].length for s in seq_ids]
            batch = build_batch(m, seq_ids, [1] * len(seq_ids), starts, decode=True)
            hidden = m.embed_tokens(torch.tensor(list(last_tokens), dtype=torch.int32))
            m.forward(batch, hidden)
            return m.greedy(m.head(hidden))
        g = self.decode_graph(seq_ids, width)
        self.stage_decode_inputs(g, seq_ids, last_tokens)
        g.upload()
        if g.use_graph and g.graph is None:
            g.capture()
        g.run()
        return g.download()

    def generate(self, prompts: Sequence[Sequence[int]], max_new_tokens: int,
                 width: Optional[int] = None, prefix: str = "s") -> List[List[int]]:
        m = self.model
        ids = [f"{prefix}{i}" for i in range(len(prompts))]
        longest = max(len(p) for p in prompts) + max_new_tokens
        width = width or -(-longest // BLOCK_SIZE)
        first = self.prefill(ids, prompts)
        out = [[int(t)] for t in first.cpu()]
        last = [o[0] for o in out]
        for _ in range(max_new_tokens - 1):
            nxt = self.decode(ids, last, width)
            if m.device.type == "cuda":
                torch.cuda.current_stream(m.device).synchronize()
            last = [int(t) for t in nxt]
            for o, t in zip(out, last):
                o.append(t)
        for sid in ids:
            m.kv.free_sequence(sid)
        return out
