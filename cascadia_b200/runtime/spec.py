"""Greedy speculative decoding over the paged-KV engine.

One round for every running sequence at once (batched):

1. draft up to ``k`` tokens per sequence, either with a small draft model
   (its own paged KV; the reference pairs Llama-3.1-8B with Llama-3.2-1B,
   crates/cascadia-engine-openvino/src/dist_spec.rs:958-1128) or with the
   n-gram prompt-lookup table (crates/cascadia-engine-sparse-moe/src/ngram_draft.rs);
2. verify: ONE target forward over ``[pending, d1 .. dk]`` per sequence
   (a ragged multi-token batch through the prefill attention kernel), LM head
   on every row, then on one GPU a single kernel (``ops.spec_verify_fused``:
   argmax of every row, longest accepted prefix, correction token, accepted
   count and the advanced KV length), with tensor parallelism the
   vocab-parallel argmax merge followed by ``ops.spec_verify``;
3. rewind: the target's KV length is reset to the accepted prefix (paged
   blocks past it go back to the pool), the draft's likewise.  No data moves.

Every round emits ``accepted + 1`` tokens per sequence, so the output equals
plain greedy decoding of the target (the acceptance rule only keeps draft
tokens the target itself would have produced).
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch

from .. import ops
from ..models.llama import build_batch
from .generator import DecodeGraph
from .kv_cache import BLOCK_SIZE

MIN_NGRAM = 2
MAX_NGRAM = 4
DEFAULT_NGRAM_K = 8


class NGramDraft:
    """Prompt-lookup draft: maps each trailing 2..4-gram of the token history
    to the token that most recently followed it; proposes by repeatedly
    extending with the longest matching n-gram (behaviour of
    crates/cascadia-engine-sparse-moe/src/ngram_draft.rs:42-190)."""

    def __init__(self, k: int = DEFAULT_NGRAM_K):
        self.k = max(1, min(64, k))
        self.history: List[int] = []
        self.table: Dict[Tuple[int, ...], int] = {}

    def append(self, t: int):
        h = self.history
        for n in range(MIN_NGRAM, MAX_NGRAM + 1):
            if len(h) >= n:
                self.table[tuple(h[-n:])] = t
        h.append(t)

    def extend(self, tokens: Sequence[int]):
        for t in tokens:
            self.append(int(t))

    def rewind(self, n: int):
        """Drop the last n history tokens (their table entries stay)."""
        n = min(n, len(self.history))
        if n:
            del self.history[-n:]

    def _next(self, buf: List[int]) -> Optional[int]:
        for n in range(MAX_NGRAM, MIN_NGRAM - 1, -1):
            if len(buf) >= n:
                t = self.table.get(tuple(buf[-n:]))
                if t is not None:
                    return t
        return None

    def propose(self, k: Optional[int] = None) -> List[int]:
        k = self.k if k is None else k
        buf = list(self.history[-MAX_NGRAM:])
        out: List[int] = []
        for _ in range(k):
            t = self._next(buf)
            if t is None:
                break
            out.append(t)
            buf.append(t)
        return out


def count_accepted(drafts: Sequence[int], target: Sequence[int]) -> int:
    """Length of the longest prefix where the draft equals the target's pick."""
    a = 0
    for d, t in zip(drafts, target):
        if d != t:
            break
        a += 1
    return a


@dataclass
class RoundReconcile:
    history_pop: int
    kv_rewind: int
    new_tokens: int


def reconcile_after_round(k_drafts: int, accepted: int, bonus_forward_ran: bool,
                          pending_in_history: bool) -> RoundReconcile:
    """KV / history bookkeeping of one round for a sequential (one token per
    forward) spec loop: ``k_drafts`` drafts were pushed and forwarded (plus an
    optional extra forward when all were accepted).  With the pending-token
    convention the history runs one token ahead of the KV, so one slot less
    is rewound.  (Same arithmetic as
    crates/cascadia-engine-sparse-moe/src/spec_decode.rs:128-178; the batched
    verify below needs only ``kv_len = kv_len + 1 + accepted``.)"""
    assert 0 <= accepted <= k_drafts
    writes = k_drafts + (1 if bonus_forward_ran else 0)
    rewind = writes - accepted
    if pending_in_history:
        assert rewind >= 1
        rewind -= 1
    return RoundReconcile(history_pop=k_drafts - accepted, kv_rewind=rewind,
                          new_tokens=accepted + 1)


@dataclass
class SpecState:
    """One sequence under speculative decoding."""
    sid: str
    tokens: List[int]                 # prompt + generated; the last is pending
    kv_len: int                       # target tokens with KV written
    ngram: Optional[NGramDraft] = None
    generated: int = 0
    done: bool = False


@dataclass
class SpecStats:
    rounds: int = 0
    drafted: int = 0
    accepted: int = 0
    emitted: int = 0
    draft_s: float = 0.0    # host wall time in the drafter (ends with a device sync)
    verify_s: float = 0.0   # host wall time in verify_batch (ends with a device sync)

    @property
    def accept_rate(self) -> float:
        return self.accepted / self.drafted if self.drafted else 0.0


class VerifyGraph(DecodeGraph):
    """A captured verify step for B sequences of exactly T rows each (the
    usual round: every sequence drafted T-1 tokens), run as a decode step of
    B*T rows: row (b, j) is token j of sequence b at position p0+j with
    sequence length p0+j+1 over sequence b's block table.  Every row's K/V
    is written before the layer's attention runs, so row j sees exactly the
    keys up to its own position (causal), and the split-KV decode attention
    kernel serves the verify (the rows of one sequence re-read the same
    blocks, from L2).  After the LM head and the argmax of every row, the
    verify kernel writes the accepted drafts, the correction token and the
    count; one D2H copy brings them back.  Plain decoding and verification
    share every kernel."""

    def __init__(self, m, B: int, T: int, W: int):
        super().__init__(m, B * T, W, use_graph=True)
        self.nseq, self.T = B, T
        dev = m.device
        # drafts [B, T-1] | KV lengths before the round [B], one H2D copy
        self.vin_host = torch.zeros(B * T, dtype=torch.int32, pin_memory=True)
        self.vin = torch.zeros(B * T, dtype=torch.int32, device=dev)
        self.draft = self.vin[:B * (T - 1)].view(B, T - 1)
        self.kv_len = self.vin[B * (T - 1):]
        self.row_seq = torch.arange(B, dtype=torch.int32, device=dev).repeat_interleave(T)
        self.row_start = torch.arange(0, (B + 1) * T, T, dtype=torch.int32, device=dev)
        self.scratch = (torch.empty(B * T, dtype=torch.int32, device=dev),
                        torch.zeros(B, dtype=torch.int32, device=dev))
        self.out = torch.empty(B, T + 1, dtype=torch.int32, device=dev)
        self.vout_host = torch.zeros(B, T + 1, dtype=torch.int32, pin_memory=True)

    def _step(self):
        m = self.model
        m.embed_tokens(self.ids, out=self.hidden)
        m.forward(self.batch_view, self.hidden)
        self.logits = m.head(self.hidden)
        if m.tp.size == 1:
            # argmax of every row + accept + correction + KV length: one kernel
            ops.spec_verify_fused(self.logits[:, :m.vocab_valid], self.row_seq, self.row_start,
                                  self.draft, self.kv_len, self.out, self.scratch)
        else:
            self.next_ids = m.greedy(self.logits)
            ops.spec_verify(self.next_ids.view(self.nseq, self.T), self.draft, self.out)
        return self.out

    def stage(self, seq_ids, rows: List[List[int]], kv_lens: List[int]):
        m, kv, B, T = self.model, self.model.kv, self.nseq, self.T
        pos = np.empty((B, T), dtype=np.int32)
        slots = np.empty((B, T), dtype=np.int32)
        table = np.zeros((B, T, self.W), dtype=np.int32)
        for i, (sid, p0) in enumerate(zip(seq_ids, kv_lens)):
            kv.reserve(sid, p0 + T)
            kv.slide(sid, m.cfg, p0)
            s = kv.seqs[sid]
            s.length = max(s.length, p0 + T)
            pos[i] = np.arange(p0, p0 + T)
            slots[i] = s.slots(p0, p0 + T)
            table[i, :, :len(s.blocks)] = np.maximum(s.blocks, 0)
        self.fill(np.asarray(rows, dtype=np.int32).reshape(-1), pos.reshape(-1),
                  slots.reshape(-1), pos.reshape(-1) + 1, table.reshape(B * T, self.W))
        v = self.vin_host.numpy()
        v[:B * (T - 1)] = np.asarray([r[1:] for r in rows], dtype=np.int32).reshape(-1)
        v[B * (T - 1):] = kv_lens
        self.upload()
        self.vin.copy_(self.vin_host, non_blocking=True)

    def verify(self) -> List[List[int]]:
        if self.graph is None:
            self.capture()
        self.run()
        self.vout_host.copy_(self.out, non_blocking=True)
        torch.cuda.current_stream(self.dev).synchronize()
        return [r[:r[-1]] for r in self.vout_host.tolist()]


def verify_batch(m, seq_ids: List[str], pending: List[int], drafts: List[List[int]],
                 kv_lens: List[int], hidden_out: Optional[list] = None,
                 graphs: Optional[dict] = None, width: int = 0) -> List[List[int]]:
    """One target forward over ``[pending, *drafts]`` per sequence (positions
    from ``kv_lens``), argmax of every row, device verify.  Returns, per
    sequence, the accepted drafts followed by the correction token.  The
    caller rewinds the KV to ``kv_len + len(result)``.  ``hidden_out``, when
    given, receives the pre-norm hidden rows of each sequence's forward.
    With ``graphs`` (a dict the caller keeps) and every sequence carrying
    the same number of drafts, the step replays a captured VerifyGraph."""
    rows = [[p] + d for p, d in zip(pending, drafts)]
    T = len(rows[0])
    if (graphs is not None and hidden_out is None and m.device.type == "cuda" and T > 1
            and T <= 64 and width > 0 and all(len(r) == T for r in rows)):
        w = -(-width // 64) * 64  # one graph for nearby table widths
        key = (len(rows), T, w)
        g = graphs.get(key)
        if g is None:
            g = graphs[key] = VerifyGraph(m, len(rows), T, w)
        g.stage(seq_ids, rows, kv_lens)
        return g.verify()
    batch = build_batch(m, seq_ids, [len(r) for r in rows], kv_lens, False)
    flat = torch.tensor([t for r in rows for t in r], dtype=torch.int32).to(m.device)
    hidden = m.embed_tokens(flat)
    m.forward(batch, hidden)
    if hidden_out is not None:
        o = 0
        for r in rows:
            hidden_out.append(hidden[o:o + len(r)])
            o += len(r)
    kmax = max(len(d) for d in drafts)
    B = len(rows)
    if m.device.type == "cuda" and m.tp.size == 1:
        # One kernel: argmax of every row, comparison with the drafts,
        # correction token, accepted count and the new KV lengths.
        logits = m.head(hidden)[:, :m.vocab_valid]
        offs = np.cumsum([0] + [len(r) for r in rows]).astype(np.int32)
        row_seq = np.repeat(np.arange(B, dtype=np.int32), [len(r) for r in rows])
        dr = np.full((B, max(kmax, 1)), -1, dtype=np.int32)
        for i, d in enumerate(drafts):
            dr[i, :len(d)] = d
        packed = torch.from_numpy(np.concatenate([offs, row_seq, dr.reshape(-1),
                                                  np.asarray(kv_lens, np.int32)]))
        dev = packed.to(m.device, non_blocking=True)
        o = 0
        row_start_t = dev[o:o + B + 1]; o += B + 1
        row_seq_t = dev[o:o + len(row_seq)]; o += len(row_seq)
        dr_t = dev[o:o + dr.size].view(B, dr.shape[1]); o += dr.size
        kvl = dev[o:o + B]
        out = torch.empty(B, dr.shape[1] + 2, dtype=torch.int32, device=m.device)
        ops.spec_verify_fused(logits, row_seq_t, row_start_t, dr_t, kvl, out)
        out = out.cpu()
        return [out[i, :int(out[i, -1])].tolist() for i in range(B)]
    picks = m.greedy(m.head(hidden)).to(torch.int32)  # argmax of every row
    if kmax == 0:
        return [[int(t)] for t in picks.cpu()]
    # Pad to [B, kmax+1] / [B, kmax] for the device verify kernel; padded
    # draft slots hold -1 and never match.
    offs = np.cumsum([0] + [len(r) for r in rows])
    tgt_idx = np.empty((B, kmax + 1), dtype=np.int64)
    dr = np.full((B, kmax), -1, dtype=np.int32)
    for i in range(B):
        n = len(rows[i])
        tgt_idx[i, :n] = np.arange(offs[i], offs[i] + n)
        tgt_idx[i, n:] = offs[i] + n - 1
        dr[i, :n - 1] = drafts[i]
    tgt = picks.index_select(0, torch.from_numpy(tgt_idx.ravel()).to(picks.device))
    tgt = tgt.view(B, kmax + 1).contiguous()
    if m.device.type == "cuda":
        out = torch.empty(B, kmax + 2, dtype=torch.int32, device=m.device)
        ops.spec_verify(tgt, torch.from_numpy(dr).to(m.device), out)
        out = out.cpu()
        return [out[i, :int(out[i, -1])].tolist() for i in range(B)]
    from ..ops import reference as ref

    t = tgt.cpu()
    return [ref.spec_verify(t[i].tolist(), drafts[i]) for i in range(B)]


class ModelDrafter:
    """Greedy drafts from a small model with its own paged KV.  Per sequence
    it remembers how many history tokens its KV holds; a round first feeds
    the unseen history tail (ragged prefill, giving d1), then k-1 decode
    steps (CUDA graphs on GPU)."""

    def __init__(self, draft, use_graph: bool = True):
        from .generator import BatchGenerator

        self.model = draft
        self.gen = BatchGenerator(draft, use_graph=use_graph)
        self.kv_len: Dict[str, int] = {}

    def propose(self, seq_ids: List[str], histories: List[List[int]], k: int,
                width: int) -> List[List[int]]:
        d = self.model
        for sid in seq_ids:
            if sid not in d.kv.seqs:
                d.kv.add_sequence(sid)
                self.kv_len[sid] = 0
        starts = [self.kv_len[sid] for sid in seq_ids]
        tails = [h[st:] for h, st in zip(histories, starts)]
        if d.device.type == "cuda" and all(len(t) == 1 for t in tails):
            # The usual round: only the last verified token is new, so the
            # first draft step is a decode step too (graph replay, no eager
            # ragged prefill).
            first = self.gen.decode(seq_ids, [t[0] for t in tails], width)
        else:
            first = self.gen.prefill(seq_ids, tails, starts)
        for sid, h in zip(seq_ids, histories):
            self.kv_len[sid] = len(h)
        drafts = [[int(t)] for t in first.cpu()]
        last = [x[0] for x in drafts]
        for _ in range(k - 1):
            nxt = self.gen.decode(seq_ids, last, width)
            if d.device.type == "cuda":
                torch.cuda.current_stream(d.device).synchronize()
            last = [int(t) for t in nxt]
            for x, t in zip(drafts, last):
                x.append(t)
        return drafts

    def accept(self, sid: str, accepted: int, k: int):
        """After verify: the draft forwarded d1 .. d_{k-1}; keep the accepted
        ones."""
        self.kv_len[sid] += min(accepted, k - 1)
        self.model.kv.truncate(sid, self.kv_len[sid])

    def release(self, sid: str):
        self.kv_len.pop(sid, None)
        if sid in self.model.kv.seqs:
            self.model.kv.free_sequence(sid)


class MTPDrafter:
    """Drafts from a multi-token-prediction head (``models.glm5.GLM5MTP``).
    The head's KV holds one row per verified position: after the prefill and
    after every verify, ``observe`` queues the new verified rows (target
    hidden, next token); ``propose`` runs them for all sequences in one
    ragged forward, whose last row per sequence gives d1, then k-1 chain
    steps (token d_i, hidden = the head's own output) give d2 .. dk.  The
    chain rows are rewound in ``accept``.  (The reference's MTP spec loop:
    crates/cascadia-engine-sparse-moe/src/glm/model.rs:404-470, one
    sequence, block KV cleared per chain.)"""

    def __init__(self, mtp):
        self.mtp = mtp
        self.kv_len: Dict[str, int] = {}
        self.queue: Dict[str, Tuple[int, List[int], List[torch.Tensor]]] = {}

    def observe(self, sid: str, start: int, next_tokens: Sequence[int], hidden: torch.Tensor):
        """Target rows at positions ``start ..`` with their pre-norm hidden
        and the verified token that follows each."""
        n = len(next_tokens)
        st, toks, hs = self.queue.get(sid, (start, [], []))
        assert st + len(toks) == start, "observed rows must be contiguous"
        self.queue[sid] = (st, toks + [int(t) for t in next_tokens], hs + [hidden[:n]])

    def propose(self, seq_ids: List[str], histories: List[List[int]], k: int,
                width: int) -> List[List[int]]:
        mtp = self.mtp
        kv = mtp.kv
        dev = mtp.device
        starts, qls, toks, hs = [], [], [], []
        for sid in seq_ids:
            if sid not in kv.seqs:
                kv.add_sequence(sid)
                self.kv_len[sid] = 0
            st, t, h = self.queue.pop(sid)
            assert st == self.kv_len[sid]
            starts.append(st)
            qls.append(len(t))
            toks.extend(t)
            hs.extend(h)
        batch = build_batch(mtp.block, seq_ids, qls, starts, False)
        ids = torch.tensor(toks, dtype=torch.int32).to(dev)
        hout, picks = mtp.step(batch, ids, torch.cat(hs).contiguous(), from_target=True)
        last = torch.tensor(batch.last_rows, dtype=torch.long, device=dev)
        h = hout.index_select(0, last).contiguous()
        d = picks.index_select(0, last)
        for sid, st, q in zip(seq_ids, starts, qls):
            self.kv_len[sid] = st + q
        drafts = [[int(t)] for t in d.cpu()]
        pos = [st + q - 1 for st, q in zip(starts, qls)]
        for _ in range(k - 1):
            pos = [p + 1 for p in pos]
            batch = build_batch(mtp.block, seq_ids, [1] * len(seq_ids), pos, True)
            h, d = mtp.step(batch, d.to(torch.int32), h, from_target=False)
            for x, t in zip(drafts, d.cpu().tolist()):
                x.append(int(t))
        return drafts

    def accept(self, sid: str, accepted: int, k: int):
        self.mtp.kv.truncate(sid, self.kv_len[sid])

    def release(self, sid: str):
        self.kv_len.pop(sid, None)
        self.queue.pop(sid, None)
        if sid in self.mtp.kv.seqs:
            self.mtp.kv.free_sequence(sid)


class SpecDecoder:
    """Batched greedy speculative decoding of `target` with either a draft
    model (``draft``: a model with its own KV cache) or n-gram drafts."""

    def __init__(self, target, draft=None, k: int = 4, ngram_k: int = DEFAULT_NGRAM_K,
                 use_graph: bool = True, mtp=None, remote_draft: bool = False):
        """With a tensor-parallel target the draft model lives on TP rank 0
        only (``draft`` given there); every other rank passes
        ``remote_draft=True`` and receives each round's drafts by a broadcast
        over the TP group (the reference's driver-side draft,
        crates/cascadia-engine-openvino/src/dist_spec.rs:958-1128)."""
        from .generator import BatchGenerator

        self.target = target
        self.remote_draft = remote_draft and draft is None
        self.share = target.tp.size > 1 and (draft is not None or self.remote_draft)
        self.k = k if (draft is not None or mtp is not None or self.remote_draft) else ngram_k
        self.tgen = BatchGenerator(target, use_graph=use_graph)
        if mtp is not None:
            self.drafter = MTPDrafter(mtp)
        else:
            self.drafter = ModelDrafter(draft, use_graph) if draft is not None else None
        self.mtp = self.drafter if mtp is not None else None
        self.stats = SpecStats()
        self.use_graph = use_graph
        self.vgraphs: Dict[tuple, VerifyGraph] = {}

    def _share_drafts(self, drafts: Optional[List[List[int]]], n: int) -> List[List[int]]:
        """Broadcast TP rank 0's drafts ([n, 1 + k] int32: length, tokens)."""
        import torch.distributed as dist

        tp = self.target.tp
        dev = self.target.device
        buf = torch.zeros(n, 1 + self.k, dtype=torch.int32)
        if drafts is not None:
            for i, d in enumerate(drafts):
                buf[i, 0] = len(d)
                buf[i, 1:1 + len(d)] = torch.tensor(d, dtype=torch.int32)
        buf = buf.to(dev)
        src = dist.get_global_rank(tp.group, 0) if tp.group is not None else 0
        dist.broadcast(buf, src, group=tp.group)
        rows = buf.cpu().tolist()
        return [r[1:1 + r[0]] for r in rows]

    def generate(self, prompts: Sequence[Sequence[int]], max_new_tokens: int,
                 eos: Sequence[int] = (), prefix: str = "spec") -> List[List[int]]:
        m = self.target
        ids = [f"{prefix}{i}" for i in range(len(prompts))]
        longest = max(len(p) for p in prompts) + max_new_tokens + self.k + 2
        width = -(-longest // BLOCK_SIZE)
        first = self.tgen.prefill(ids, prompts)
        if self.mtp is not None:
            hid, o = self.tgen.last_hidden, 0
        states = []
        for sid, p, t in zip(ids, prompts, first.cpu().tolist()):
            s = SpecState(sid, list(p) + [int(t)], kv_len=len(p), generated=1)
            if self.mtp is not None:
                self.mtp.observe(sid, 0, list(p[1:]) + [int(t)], hid[o:o + len(p)])
                o += len(p)
            if self.drafter is None and not self.remote_draft:
                s.ngram = NGramDraft(self.k)
                s.ngram.extend(s.tokens)
            s.done = max_new_tokens <= 1 or int(t) in eos
            states.append(s)
        while True:
            live = [s for s in states if not s.done]
            if not live:
                break
            t0 = time.perf_counter()
            if self.drafter is not None:
                drafts = self.drafter.propose([s.sid for s in live], [s.tokens for s in live],
                                              self.k, width)
            elif self.remote_draft:
                drafts = None
            else:
                drafts = [s.ngram.propose(self.k) for s in live]
            if self.share:
                drafts = self._share_drafts(drafts, len(live))
            # Never draft past the token budget.
            drafts = [d[:max(0, max_new_tokens - s.generated - 1)] for s, d in zip(live, drafts)]
            hid = [] if self.mtp is not None else None
            t1 = time.perf_counter()
            accepted = verify_batch(m, [s.sid for s in live], [s.tokens[-1] for s in live],
                                    drafts, [s.kv_len for s in live], hid,
                                    self.vgraphs if self.use_graph else None, width)
            self.stats.draft_s += t1 - t0
            self.stats.verify_s += time.perf_counter() - t1
            self.stats.rounds += 1
            for i, (s, d, acc) in enumerate(zip(live, drafts, accepted)):
                a = len(acc) - 1
                if self.mtp is not None:
                    # Rows kv_len .. kv_len + a are verified; each is followed
                    # by the next accepted token (the last by the correction).
                    self.mtp.observe(s.sid, s.kv_len, acc, hid[i])
                self.stats.drafted += len(d)
                self.stats.accepted += a
                new = acc[:max_new_tokens - s.generated]
                for j, t in enumerate(new):
                    if t in eos:
                        new = new[:j + 1]
                        break
                s.kv_len += 1 + a
                m.kv.truncate(s.sid, s.kv_len)
                if self.drafter is not None:
                    self.drafter.accept(s.sid, a, self.k)
                s.tokens.extend(new)
                if s.ngram is not None:
                    s.ngram.extend(new)
                s.generated += len(new)
                self.stats.emitted += len(new)
                if s.generated >= max_new_tokens or (new and new[-1] in eos):
                    s.done = True
        out = []
        for s, p in zip(states, prompts):
            out.append(s.tokens[len(p):])
            m.kv.free_sequence(s.sid)
            if self.drafter is not None:
                self.drafter.release(s.sid)
        return out
