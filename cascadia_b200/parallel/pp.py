"""Pipeline parallelism: stage relay for the dense engine.

Protocol (one engine iteration):

* rank 0 (first stage) owns the scheduler, tokenizer and API.  It runs its
  layers for the iteration's batch and sends ``meta`` (int32) + ``hidden``
  ([T, H] bf16) downstream;
* a middle stage receives, rebuilds the batch from ``meta`` (positions, KV
  slots, block tables: block ids are decided by rank 0, every stage's KV pool
  has the same number of blocks), runs its layers and forwards;
* the last stage runs its layers, the final norm and the LM head, picks greedy
  tokens on device and replies ``[seq, n, tokens...]`` upstream (plus the
  logits of rows that need sampling, which rank 0 samples with the request's
  history).  Replies travel back through the chain.

The reply echoes the iteration's sequence number; a mismatch aborts the batch
(``BatchAborted``) instead of mis-assigning tokens, as the reference's seq echo
does (crates/cascadia-engine-openvino/src/runtime.rs:950).  ``RESET`` drops all
per-sequence state downstream.  Wire kinds mirror the reference's stage
protocols (FORWARD / RESET, crates/cascadia-engine-sparse-moe/src/dist.rs:82-138).

Transports: :class:`TcpChannel` (native TCP frames, CPU / loopback — the
BASELINE 2-stage CPU config) and :class:`NcclChannel` (NCCL p2p send/recv
between GPU ranks over NVLink).
"""
from __future__ import annotations

import itertools
from typing import List, Optional, Tuple

import numpy as np
import torch

from ..engine.base import BatchAborted, Engine, EngineError, ShutdownRequested
from ..models.llama import Batch
from .. import ops

KIND_FORWARD = 1
KIND_RESET = 3
KIND_SHUTDOWN = 9
HDR = 8


def encode_meta(kind: int, seq: int, batch: Optional[Batch], want_logits: List[int]) -> torch.Tensor:
    if batch is None:
        return torch.tensor([kind, seq, 0, 0, 0, 0, 0, 0], dtype=torch.int32)
    B = len(batch.q_lens)
    T = int(batch.positions.numel())
    W = int(batch.block_tables.shape[1])
    parts = [np.array([kind, seq, B, T, int(batch.is_decode), W, len(want_logits), 0], np.int32),
             np.asarray(batch.q_lens, np.int32), np.asarray(batch.ctx_lens, np.int32),
             batch.positions.cpu().numpy().astype(np.int32),
             batch.slots.cpu().numpy().astype(np.int32),
             batch.block_tables.cpu().numpy().astype(np.int32).reshape(-1),
             np.asarray(want_logits, np.int32)]
    return torch.from_numpy(np.concatenate(parts))


def decode_meta(meta: torch.Tensor, model) -> Tuple[int, int, Optional[Batch], List[int]]:
    m = meta.cpu().numpy().astype(np.int64)
    kind, seq, B, T, dec, W, nl = (int(x) for x in m[:7])
    if kind != KIND_FORWARD:
        return kind, seq, None, []
    o = HDR
    q_lens = m[o:o + B].tolist(); o += B
    ctx = m[o:o + B].tolist(); o += B
    pos = m[o:o + T]; o += T
    slots = m[o:o + T]; o += T
    table = m[o:o + B * W].reshape(B, W); o += B * W
    want = m[o:o + nl].tolist()
    dev = model.device
    b = Batch(seq_ids=[f"r{i}" for i in range(B)], q_lens=q_lens, ctx_lens=ctx,
              positions=torch.tensor(pos, dtype=torch.int32, device=dev),
              slots=torch.tensor(slots, dtype=torch.int32, device=dev),
              block_tables=torch.tensor(table, dtype=torch.int32, device=dev),
              seq_lens=torch.tensor(ctx, dtype=torch.int32, device=dev), is_decode=bool(dec))
    if dev.type == "cuda":
        if b.is_decode:
            b.num_splits, b.blocks_per_split = ops.decode_split_plan(B, model.hkv, W)
            g = model.hq // model.hkv
            n = B * model.hkv * b.num_splits * g
            b.part_o = torch.empty(n * model.d, dtype=torch.float32, device=dev)
            b.part_ml = torch.empty(n * 2, dtype=torch.float32, device=dev)
        else:
            b.tiles = ops.prefill_tiles(q_lens, ctx, dev)
    else:
        # CPU oracle path gathers K/V per sequence through the block table.
        kv = model.kv
        from ..runtime.kv_cache import SeqKV

        for i, sid in enumerate(b.seq_ids):
            nb = -(-ctx[i] // 16)
            kv.seqs[sid] = SeqKV(blocks=[int(x) for x in table[i, :nb]], length=ctx[i])
    return kind, seq, b, want


# ----------------------------------------------------------------- channels
class TcpChannel:
    """Stage links over the native TCP transport (tensor frames)."""

    def __init__(self, up=None, down=None, reply_wait_s: float = 120.0):
        self.up, self.down = up, down
        self.reply_wait_s = reply_wait_s

    def send_down(self, meta, hidden):
        self.down.send(meta)
        if hidden is not None:
            self.down.send(hidden)

    def recv_up(self):
        meta = self.up.recv().reshape(-1)  # waits up to the idle ceiling for a frame
        hidden = None
        if int(meta[0]) == KIND_FORWARD:
            h = self.up.recv()
            hidden = h.reshape(int(meta[3]), -1)
        return meta, hidden

    def send_reply_up(self, reply, logits):
        self.up.send(reply)
        if logits is not None:
            self.up.send(logits)

    def recv_reply_down(self, with_logits: bool):
        reply = self.down.recv(first_byte_s=self.reply_wait_s).reshape(-1)
        logits = None
        if with_logits:
            logits = self.down.recv()
            logits = logits.reshape(int(reply[-1]), -1)
        return reply, logits

    def close(self):
        for l in (self.up, self.down):
            if l is not None:
                l.close()


class NcclChannel:
    """Stage links over NCCL p2p (GPU ranks of one process group).

    Frames: a 1-element length, then the tensor (shapes come from meta)."""

    def __init__(self, rank: int, world: int, device, hidden_size: int, group=None):
        self.rank, self.world = rank, world
        self.dev = torch.device(device)
        self.h = hidden_size
        self.group = group
        self.prev = rank - 1 if rank > 0 else None
        self.next = rank + 1 if rank < world - 1 else None

    def _send(self, t, dst):
        torch.distributed.send(t.contiguous(), dst, group=self.group)

    def _recv(self, shape, dtype, src):
        t = torch.empty(shape, dtype=dtype, device=self.dev)
        torch.distributed.recv(t, src, group=self.group)
        return t

    def send_down(self, meta, hidden):
        m = meta.to(self.dev)
        self._send(torch.tensor([m.numel()], dtype=torch.int32, device=self.dev), self.next)
        self._send(m, self.next)
        if hidden is not None:
            self._send(hidden, self.next)

    def recv_up(self):
        n = int(self._recv([1], torch.int32, self.prev)[0])
        meta = self._recv([n], torch.int32, self.prev).cpu()
        hidden = None
        if int(meta[0]) == KIND_FORWARD:
            hidden = self._recv([int(meta[3]), self.h], torch.bfloat16, self.prev)
        return meta, hidden

    def send_reply_up(self, reply, logits):
        r = reply.to(self.dev)
        self._send(torch.tensor([r.numel(), 0 if logits is None else logits.shape[1]],
                                dtype=torch.int32, device=self.dev), self.prev)
        self._send(r, self.prev)
        if logits is not None:
            self._send(logits.float(), self.prev)

    def recv_reply_down(self, with_logits: bool):
        hdr = self._recv([2], torch.int32, self.next).cpu()
        reply = self._recv([int(hdr[0])], torch.int32, self.next).cpu()
        logits = None
        if int(hdr[1]) > 0:
            logits = self._recv([int(reply[-1]), int(hdr[1])], torch.float32, self.next)
        return reply, logits

    def close(self):
        pass


# ----------------------------------------------------------------- stages
def make_reply(seq: int, tokens: List[int], want: List[int]) -> torch.Tensor:
    return torch.tensor([seq, len(tokens)] + list(tokens) + [len(want)], dtype=torch.int32)


class PipelineWorker(Engine):
    """A stage other than the first: relay loop body (one frame per step)."""

    def __init__(self, model, channel, is_last: bool):
        self.model = model
        self.ch = channel
        self.is_last = is_last
        self.closed = False

    def submit(self, task) -> None:
        raise EngineError("pipeline workers do not accept tasks")

    def step(self):
        meta, hidden = self.ch.recv_up()
        kind, seq, batch, want = decode_meta(meta, self.model)
        if kind == KIND_SHUTDOWN:
            if not self.is_last:
                self.ch.send_down(meta, None)
            self.closed = True
            raise ShutdownRequested()
        if kind == KIND_RESET:
            if self.model.kv is not None:
                self.model.kv.seqs.clear()
            if not self.is_last:
                self.ch.send_down(meta, None)
            return []
        m = self.model
        buf = hidden.to(m.device)
        hidden = m.unpack_payload(buf, batch, out=torch.empty(
            buf.shape[0], m.cfg.hidden_size, dtype=buf.dtype, device=m.device))
        self.model.forward(batch, hidden)
        if not self.is_last:
            self.ch.send_down(meta, m.pack_payload(hidden, batch))
            reply, logits = self.ch.recv_reply_down(bool(want))
            self.ch.send_reply_up(reply, logits)
        else:
            rows = torch.tensor(batch.last_rows, dtype=torch.long, device=self.model.device)
            logits = self.model.head(hidden.index_select(0, rows).contiguous())
            toks = [int(t) for t in self.model.greedy(logits).tolist()]
            full = self.model.full_logits(logits)[want].float() if want else None
            self.ch.send_reply_up(make_reply(seq, toks, want), full)
        if self.model.device.type == "cpu":
            self.model.kv.seqs.clear()
        return []

    def has_work(self) -> bool:
        return not self.closed


class PipelineHead:
    """First-stage side of the relay, used by the LLM engine's forward hook."""

    def __init__(self, model, channel):
        self.model = model
        self.ch = channel
        self._seq = itertools.count(1)

    def forward_tokens(self, batch: Batch, hidden: torch.Tensor, want: List[int]):
        """Run this stage, ship downstream, return (tokens, logits_for_want)."""
        seq = next(self._seq)
        self.model.forward(batch, hidden)
        meta = encode_meta(KIND_FORWARD, seq, batch, want)
        self.ch.send_down(meta, self.model.pack_payload(hidden, batch))
        reply, logits = self.ch.recv_reply_down(bool(want))
        r = reply.tolist()
        if r[0] != seq:
            raise BatchAborted(f"reply for step {r[0]} while waiting for step {seq}")
        n = r[1]
        return r[2:2 + n], logits

    def reset(self):
        self.ch.send_down(encode_meta(KIND_RESET, 0, None, []), None)

    def shutdown(self):
        try:
            self.ch.send_down(encode_meta(KIND_SHUTDOWN, 0, None, []), None)
        except EngineError:
            pass
