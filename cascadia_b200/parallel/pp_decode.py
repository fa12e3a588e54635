"""Pipelined decode across stages with micro-batch overlap.

Every rank holds one contiguous layer range (stage s of S) and the same
sequences' KV bookkeeping (block ids are allocated identically on every
stage).  The running batch is split into M micro-batches; each decode step
runs micro-batch after micro-batch:

    stage 0:   tokens(mb) --> embed + layers --> isend hidden to stage 1
    stage s:   irecv hidden <-- stage s-1; layers; isend to stage s+1
    stage S-1: irecv hidden; layers; head + argmax; isend tokens to stage 0

The sends and receives are asynchronous point-to-point operations (NCCL on
GPUs: they run on NCCL's own streams, ordered against the compute stream by
events), so while stage s computes micro-batch m+1, micro-batch m is on the
wire and stage s+1 computes it.  With M >= S the pipeline stays full: the
tokens of micro-batch m return to stage 0 before it comes round to m again.
The next tokens never go through the host: stage 0 receives them straight
into the input buffer of the micro-batch's CUDA graph.  Each micro-batch
step of a stage is one CUDA graph replay.

This is the B200 counterpart of the reference's relay of hidden rows
between stages over TCP (crates/cascadia-engine-openvino/src/runtime.rs:3312-3400),
which runs one request step at a time with no overlap.
"""
from __future__ import annotations

from typing import List, Sequence

import numpy as np
import torch
import torch.distributed as dist

from ..runtime.generator import DecodeGraph
from ..runtime.kv_cache import BLOCK_SIZE


class PipelinedDecoder:
    def __init__(self, model, stage: int, n_stages: int, micro_batches: List[List[str]],
                 width: int, group=None, ranks: Sequence[int] = None, use_graph: bool = True):
        self.m = model
        self.stage, self.S = stage, n_stages
        self.mbs = micro_batches
        self.W = width
        self.group = group
        self.ranks = list(ranks) if ranks is not None else list(range(n_stages))
        self.graphs = [DecodeGraph(model, len(ids), width, use_graph) for ids in micro_batches]
        self._pending: List[list] = [[] for _ in micro_batches]  # sends reading graph buffers
        self.first = stage == 0
        self.last = stage == n_stages - 1

    def _peer(self, s: int) -> int:
        return self.ranks[s]

    def _stage_inputs(self, g: DecodeGraph, ids: List[str]):
        kv = self.m.kv
        b = len(ids)
        pos = np.empty(b, np.int32)
        slots = np.empty(b, np.int32)
        lens = np.empty(b, np.int32)
        table = np.zeros((b, g.W), np.int32)
        for i, sid in enumerate(ids):
            s = kv.seqs[sid]
            p = s.length
            kv.reserve(sid, p + 1)
            s.length = p + 1
            pos[i] = p
            slots[i] = s.blocks[p // BLOCK_SIZE] * BLOCK_SIZE + p % BLOCK_SIZE
            lens[i] = p + 1
            kv.slide(sid, self.m.cfg, p)
            table[i, :len(s.blocks)] = np.maximum(s.blocks, 0)
        # ids arrive by p2p (stage 0) or are unused: keep what is in the buffer.
        g.fill(g.host.numpy()[:b].copy(), pos, slots, lens, table)
        # The CPU oracle attention looks sequences up by id.
        g.batch_view.seq_ids = list(ids)
        g.batch_view.ctx_lens = [int(x) for x in lens]

    def set_tokens(self, mb: int, tokens):
        """Stage 0: the first tokens of a micro-batch (from the prefill)."""
        g = self.graphs[mb]
        g.ids.copy_(torch.as_tensor(np.asarray(tokens, np.int32)).to(g.ids.device))
        g.host.numpy()[:len(tokens)] = tokens

    def step(self, capture_now: bool = False):
        """One decode step of every micro-batch through this stage."""
        for mb, ids in enumerate(self.mbs):
            g = self.graphs[mb]
            for w in self._pending[mb]:
                w.wait()
            self._pending[mb] = []
            self._stage_inputs(g, ids)
            # Upload positions / slots / table, but keep the received ids.
            b = g.B
            g.dev_in[b:].copy_(g.host[b:], non_blocking=True)
            if not self.first:
                dist.irecv(g.hidden_in, self._peer(self.stage - 1), group=self.group).wait()
            if g.use_graph and g.graph is None and capture_now:
                g.capture()
            g.run()
            if not self.last:
                self._pending[mb].append(
                    dist.isend(g.payload_out, self._peer(self.stage + 1), group=self.group))
            else:
                self._pending[mb].append(
                    dist.isend(g.next_ids.to(torch.int32), self._peer(0), group=self.group))
            if self.first and self.S > 1:
                # Next step's tokens of this micro-batch come back from the
                # last stage straight into the graph's input ids.
                self._pending[mb].append(
                    dist.irecv(g.ids, self._peer(self.S - 1), group=self.group))
            elif self.first:
                g.ids.copy_(g.next_ids)

    def finish(self):
        for lst in self._pending:
            for w in lst:
                w.wait()
        self._pending = [[] for _ in self.mbs]

    def tokens(self, mb: int) -> List[int]:
        """Stage 0 after finish(): the latest tokens of a micro-batch."""
        return [int(t) for t in self.graphs[mb].ids.cpu()]


def pp_prefill(model, stage: int, n_stages: int, seq_ids: List[str], prompts: List[List[int]],
               group=None, ranks: Sequence[int] = None) -> List[int]:
    """Prefill a group of sequences through the stages (blocking hand-off of
    the hidden rows, as the prompt needs every layer before the first token).
    Returns the first tokens on stage 0 (an empty list elsewhere)."""
    from ..models.llama import build_batch

    ranks = list(ranks) if ranks is not None else list(range(n_stages))
    m = model
    for sid in seq_ids:
        if sid not in m.kv.seqs:
            m.kv.add_sequence(sid)
    batch = build_batch(m, seq_ids, [len(p) for p in prompts], [0] * len(prompts), False)
    T = sum(len(p) for p in prompts)
    if stage == 0:
        hidden = m.embed_tokens(torch.tensor([t for p in prompts for t in p], dtype=torch.int32,
                                             device=m.device))
    else:
        buf = torch.empty(T, m.payload_in_width, dtype=torch.bfloat16, device=m.device)
        dist.recv(buf, ranks[stage - 1], group=group)
        hidden = m.unpack_payload(buf, batch,
                                  out=torch.empty(T, m.cfg.hidden_size, dtype=torch.bfloat16,
                                                  device=m.device))
    m.forward(batch, hidden)
    if stage < n_stages - 1:
        dist.send(m.pack_payload(hidden, batch).contiguous(), ranks[stage + 1], group=group)
    else:
        rows = torch.tensor(batch.last_rows, dtype=torch.long, device=m.device)
        toks = m.greedy(m.head(hidden.index_select(0, rows).contiguous())).to(torch.int32)
        if n_stages > 1:
            dist.send(toks, ranks[0], group=group)
        else:
            return [int(t) for t in toks.cpu()]
    if stage == 0:
        toks = torch.empty(len(prompts), dtype=torch.int32, device=m.device)
        dist.recv(toks, ranks[n_stages - 1], group=group)
        return [int(t) for t in toks.cpu()]
    return []
