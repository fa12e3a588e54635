"""The dense GPU serving engine (Llama-family INT4), single stage.

This is the B200 counterpart of the reference's ``ov-runtime`` /
``ov-genai --cb`` engines (crates/cascadia-engine-openvino/src/runtime.rs,
genai.rs:597-915): one ``step()`` = one continuous-batching iteration:

1. admit waiting requests and run one chunked-prefill pass (packed ragged
   prompts, paged KV, prefix-cache hits skipped);
2. run one decode step for every running sequence through a captured CUDA
   graph (batch padded to a bucket: padded rows write no KV);
3. pick tokens on device (greedy argmax in the graph, or the sampling kernel
   for rows with temperature > 0), detokenize incrementally, finish on EOS /
   ``max_tokens``, free KV.

Chunks follow the reference conventions: one token chunk per generated token,
``prompt_tokens`` on the final chunk, ``finish_reason`` stop/length.
"""
from __future__ import annotations

import logging
import math
import time
from typing import Dict, Iterable, List, Optional

import numpy as np
import torch

from .. import metrics, ops
from ..api.templates import ByteTokenizer, IncrementalDecoder
from ..models.llama import build_batch
from ..ops import reference as ref
from ..runtime.generator import DecodeGraph
from ..runtime.kv_cache import BLOCK_SIZE
from ..runtime.scheduler import PrefixCache, SchedulerState, Sequence
from ..utils.trace import span, task_done
from ..types import (Chunk, FinishReason, GenerationTask, LoadProgress, PeerLayout, ShardSpec,
                     TokenLogprobs, TopLogprob)
from .base import (BatchAborted, Builder, Engine, EngineError, InvalidConfig, NotLoaded,
                   PromptTooLong, QueueFull)

log = logging.getLogger("cascadia.engine")

BATCH_BUCKETS = (1, 2, 4, 8, 16, 32, 64, 128, 256)


def _bucket(n: int, buckets=BATCH_BUCKETS) -> int:
    for b in buckets:
        if n <= b:
            return b
    return n


class LLMEngine(Engine):
    def __init__(self, model, tokenizer=None, max_running: int = 64,
                 max_prefill_tokens: int = 8192, max_model_len: int = 8192,
                 use_graph: bool = True, prefix_cache_blocks: int = 0, model_id: str = "llm",
                 max_queue: int = 1024, spec: Optional[str] = None, draft_model=None,
                 spec_k: int = 4, mtp_head=None):
        self.model = model
        self.dev = model.device
        self.cfg = model.cfg
        self.tok = tokenizer or ByteTokenizer(vocab_size=model.cfg.vocab_size,
                                              eos_id=model.cfg.eos_token_ids[0])
        self.eos = set(model.cfg.eos_token_ids)
        if getattr(self.tok, "eos_id", None) is not None:
            self.eos.add(self.tok.eos_id)
        self.max_model_len = max_model_len
        self.max_queue = max_queue
        pc = PrefixCache(model.kv, f"{model_id}", prefix_cache_blocks) \
            if prefix_cache_blocks > 0 else None
        self.sched = SchedulerState(model.kv, max_running, max_prefill_tokens, pc, max_queue)
        self.use_graph = use_graph and self.dev.type == "cuda"
        self.graphs: Dict[tuple, DecodeGraph] = {}
        self.decoders: Dict[str, IncrementalDecoder] = {}
        self.model_id = model_id
        self._seq_counter = 0
        self.last_step_ms = 0.0
        self.aborted_batches = 0
        self._pending_lp: Dict[str, TokenLogprobs] = {}
        # Set for the first stage of a pipeline (parallel.pp.PipelineHead):
        # the model forward then relays through the downstream stages.
        self.pipeline = None
        # Speculative decoding of greedy sequences: "ngram" (prompt lookup),
        # "draft" (a small model with its own KV, ``draft_model``) or "mtp"
        # (a GLM-5 multi-token-prediction head, ``mtp_head``).
        if spec not in (None, "ngram", "draft", "mtp"):
            raise InvalidConfig(f"unknown speculative mode {spec!r}")
        if spec == "draft" and draft_model is None:
            raise InvalidConfig("speculative mode 'draft' needs a draft model")
        if spec == "mtp" and (mtp_head is None or pc is not None):
            # The head reads the target's hidden row of every prompt token,
            # which a prefix-cache hit skips.
            raise InvalidConfig("speculative mode 'mtp' needs an MTP head and no prefix cache")
        self.spec = spec
        self.spec_k = spec_k
        self.drafter = None
        if spec == "draft":
            from ..runtime.spec import ModelDrafter

            self.drafter = ModelDrafter(draft_model, use_graph)
        elif spec == "mtp":
            from ..runtime.spec import MTPDrafter

            self.drafter = MTPDrafter(mtp_head)
        self.spec_stats = None
        if spec is not None:
            from ..runtime.spec import SpecStats

            self.spec_stats = SpecStats()

    # ------------------------------------------------------------ Engine API
    def warmup(self) -> None:
        if self.dev.type != "cuda":
            return
        t = GenerationTask("__warmup__", "warm", max_tokens=2, prompt_ids=[1, 2, 3, 4])
        self.submit(t)
        for _ in range(8):
            out = self.step()
            if any(c.is_final for _, c in out):
                break
        self.cancel("__warmup__")
        torch.cuda.synchronize(self.dev)

    def has_work(self) -> bool:
        return bool(self.sched.waiting or self.sched.running)

    def submit(self, task: GenerationTask) -> None:
        if task.task_id in self.sched.by_id:
            return
        if len(self.sched.waiting) >= self.max_queue:
            raise QueueFull(len(self.sched.waiting), self.max_queue)
        ids = list(task.prompt_ids) if task.prompt_ids else self.tok.encode(task.prompt)
        if not ids:
            ids = [0]
        if any(i < 0 or i >= self.cfg.vocab_size for i in ids):
            raise InvalidConfig("prompt token id out of range")
        if len(ids) + 1 > self.max_model_len:
            raise PromptTooLong(f"{len(ids)} tokens > window {self.max_model_len - 1}")
        blocks_needed = -(-(len(ids) + 1) // BLOCK_SIZE)
        if blocks_needed > self.model.kv.num_blocks:
            raise PromptTooLong(f"{len(ids)} tokens exceed the KV cache")
        seq = Sequence(task=task, prompt_ids=ids, seq_id=task.task_id)
        seq.submitted_at = time.monotonic()
        self.sched.add(seq)
        self.decoders[task.task_id] = IncrementalDecoder(self.tok)

    def cancel(self, task_id: str) -> None:
        self.sched.remove(task_id)
        self.decoders.pop(task_id, None)
        if self.drafter is not None:
            self.drafter.release(task_id)

    def close(self) -> None:
        for sid in list(self.sched.by_id):
            self.cancel(sid)
        self.graphs.clear()

    def step(self) -> List[tuple]:
        out: List[tuple] = []
        t0 = time.perf_counter()
        work = self.sched.admit()
        if work:
            with span("prefill"):
                self._prefill(work, out)
            metrics.STEP_SECONDS.labels(model=self.model_id, phase="prefill").observe(
                time.perf_counter() - t0)
        dec = self.sched.decode_set()
        # Sequences whose first token came from this step's prefill (or that
        # it aborted) are not decoded again in the same iteration.
        just = {s.seq_id for s, st, n in work}
        dec = [s for s in dec if s.seq_id not in just]
        if dec:
            t1 = time.perf_counter()
            with span("decode"):
                self._decode(dec, out)
            metrics.STEP_SECONDS.labels(model=self.model_id, phase="decode").observe(
                time.perf_counter() - t1)
        self.last_step_ms = (time.perf_counter() - t0) * 1000
        kv = self.model.kv
        metrics.KV_BLOCKS_USED.labels(model=self.model_id).set(
            kv.num_blocks - kv.allocator.num_free)
        metrics.KV_BLOCKS_TOTAL.labels(model=self.model_id).set(kv.num_blocks)
        return out

    # ------------------------------------------------------------ device status
    def _device_failed(self, seqs: List[Sequence], out) -> bool:
        """Read the device status word after a forward (a few bytes, on the
        same stream the forward ran on).  A bounded wait inside a kernel that
        gave up (a peer that never signalled, a copy that never landed)
        leaves its outputs unwritten and sets this word: the batch that ran
        is then failed with an error chunk per sequence, its KV freed, and
        the engine keeps serving the next requests (the reference's
        BatchAborted, crates/cascadia-engine/src/lib.rs:56-72)."""
        code = ops.read_status(self.dev)
        tp = getattr(self.model, "tp", None)
        ep = getattr(self.model, "ep", None)
        tp_on = tp is not None and tp.size > 1
        ep_on = ep is not None and ep.world > 1
        group = tp.group if tp_on else (ep.group if ep_on else None)
        if tp_on or ep_on:
            # Every replica must fail the same batch: the worst status of the
            # TP (or EP) ranks decides (one tiny collective per iteration).
            t = torch.tensor([code], dtype=torch.int32,
                             device=self.dev if self.dev.type == "cuda" else "cpu")
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX, group=group)
            code = int(t.item())
        if code == 0:
            return False
        err = BatchAborted(f"device status {code} ({ops.status_name(code)})")
        log.error("%s: failing %d sequence(s)", err, len(seqs))
        self.aborted_batches += 1
        for s in seqs:
            if s.finished:
                continue
            s.finished = True
            tid = s.task.task_id
            out.append((tid, Chunk.error_chunk(tid, str(err))))
            if self.drafter is not None:
                self.drafter.release(s.seq_id)
            self.sched.remove(s.seq_id)
            self.decoders.pop(tid, None)
        return True

    # ------------------------------------------------------------ prefill
    def _prefill(self, work, out):
        m = self.model
        seq_ids = [s.seq_id for s, _, _ in work]
        q_lens = [n for _, _, n in work]
        starts = [st for _, st, _ in work]
        batch = build_batch(m, seq_ids, q_lens, starts, decode=False)
        ids = torch.tensor([t for s, st, n in work for t in s.prompt_ids[st:st + n]],
                           dtype=torch.int32).to(self.dev, non_blocking=True)
        for s, st, n in work:
            s.prefilled = st + n
        seqs = [s for s, _, _ in work]
        toks = self._run_model(batch, ids, seqs)
        if self._device_failed(seqs, out):
            return
        if self.spec == "mtp" and self.pipeline is None:
            # Queue every prompt row of a greedy sequence (the ones that
            # decode speculatively) for the MTP head, with the token after it.
            off = 0
            for (s, st, n), t in zip(work, toks):
                if s.task.temperature <= 0 and not self._has_penalty(s):
                    p = s.prompt_ids
                    nxt = list(p[st + 1:st + n]) + [p[st + n] if st + n < len(p) else int(t)]
                    self.drafter.observe(s.seq_id, st, nxt, self._last_hidden[off:off + n])
                off += n
        lps = getattr(self, "_pending_lp", {})
        for s, t in zip(seqs, toks):
            if not s.in_prefill:
                self._emit(s, int(t), out, lps.get(s.seq_id))
        self._pending_lp = {}

    def _run_model(self, batch, ids, seqs: List[Sequence]) -> List[int]:
        """Forward the batch and pick one token per sequence (its last row)."""
        m = self.model
        hidden = m.embed_tokens(ids)
        if self.pipeline is None:
            m.forward(batch, hidden)
            self._last_hidden = hidden
            rows = torch.tensor(batch.last_rows, dtype=torch.long, device=self.dev)
            logits = m.head(hidden.index_select(0, rows).contiguous())
            toks = self._pick(seqs, logits)
            self._pending_lp = self._logprobs(
                [(i, s) for i, s in enumerate(seqs) if not s.in_prefill], logits, toks)
            return toks
        # Rows whose full logits come back from the last stage: sampled
        # rows, and rows whose task asked for logprobs.
        want = [i for i, s in enumerate(seqs)
                if not s.in_prefill and (s.task.temperature > 0 or self._has_penalty(s)
                                         or s.task.logprobs > 0)]
        toks, logits = self.pipeline.forward_tokens(batch, hidden, want)
        toks = list(toks)
        if want:
            logits = logits.to(self.dev)
            samp = [k for k, i in enumerate(want)
                    if seqs[i].task.temperature > 0 or self._has_penalty(seqs[i])]
            if samp:
                picked = self._pick_full([seqs[want[k]] for k in samp],
                                         logits.index_select(0, torch.tensor(
                                             samp, dtype=torch.long, device=self.dev)))
                for k, t in zip(samp, picked):
                    toks[want[k]] = t
            self._pending_lp = self._logprobs([(k, seqs[i]) for k, i in enumerate(want)],
                                              logits, [toks[i] for i in want])
        return toks

    # ------------------------------------------------------------ decode
    def _graph_for(self, b: int, width: int) -> DecodeGraph:
        key = (b, width)
        g = self.graphs.get(key)
        if g is None:
            g = DecodeGraph(self.model, b, width, self.use_graph)
            self.graphs[key] = g
        return g

    def _decode(self, seqs: List[Sequence], out):
        m = self.model
        kv = m.kv
        if self.spec is not None and self.pipeline is None:
            greedy = [s for s in seqs if self._speculable(s)]
            if greedy:
                self._spec_decode(greedy, out)
                seqs = [s for s in seqs if not self._speculable(s)]
                if not seqs:
                    return
        if self.dev.type != "cuda" or self.pipeline is not None:
            starts = [s.total_len - 1 for s in seqs]
            batch = build_batch(m, [s.seq_id for s in seqs], [1] * len(seqs), starts, True)
            ids = torch.tensor([s.output_ids[-1] for s in seqs], dtype=torch.int32).to(self.dev)
            toks = self._run_model(batch, ids, seqs)
            if self._device_failed(seqs, out):
                return
            lps = getattr(self, "_pending_lp", {})
            self._pending_lp = {}
            for s, t in zip(seqs, toks):
                self._emit(s, int(t), out, lps.get(s.seq_id))
            return
        n = len(seqs)
        B = _bucket(n)
        maxlen = max(s.total_len for s in seqs) + 1
        width = 1 << max(4, math.ceil(math.log2(-(-maxlen // BLOCK_SIZE))))
        g = self._graph_for(B, width)
        ids = np.zeros(B, np.int32)
        pos = np.zeros(B, np.int32)
        slots = np.full(B, -1, np.int32)
        lens = np.zeros(B, np.int32)
        table = np.zeros((B, width), np.int32)
        for i, s in enumerate(seqs):
            kv.reserve(s.seq_id, s.total_len)
            st = kv.seqs[s.seq_id]
            p = s.total_len - 1  # position of the token being fed
            st.length = p + 1
            ids[i] = s.output_ids[-1]
            pos[i] = p
            slots[i] = st.blocks[p // BLOCK_SIZE] * BLOCK_SIZE + p % BLOCK_SIZE
            lens[i] = p + 1
            kv.slide(s.seq_id, self.model.cfg, p)
            table[i, :len(st.blocks)] = np.maximum(st.blocks, 0)
        g.fill(ids, pos, slots, lens, table)
        g.upload()
        if g.use_graph and g.graph is None:
            g.capture()
        g.run()
        if all(s.task.temperature <= 0 and not self._has_penalty(s) for s in seqs):
            g.download()
            torch.cuda.current_stream(self.dev).synchronize()
            toks = [int(t) for t in g.out_host[:n]]
        else:
            toks = self._pick(seqs, g.logits[:n])
        if self._device_failed(seqs, out):
            return
        lps = self._logprobs(list(enumerate(seqs)), g.logits[:n], toks)
        for s, t in zip(seqs, toks):
            self._emit(s, int(t), out, lps.get(s.seq_id))

    def _spec_decode(self, seqs: List[Sequence], out):
        """One speculative round for greedy sequences: draft, verify in one
        multi-token target forward, emit the accepted tokens + correction,
        rewind the KV to the accepted prefix."""
        from ..runtime.spec import NGramDraft, verify_batch

        m = self.model
        k = self.spec_k
        budget = [max(0, min(s.task.max_tokens - len(s.output_ids),
                             self.max_model_len - s.total_len - 1) - 1) for s in seqs]
        ids = [s.seq_id for s in seqs]
        if self.drafter is not None:
            maxlen = max(s.total_len for s in seqs) + k + 1
            width = 1 << max(4, math.ceil(math.log2(-(-maxlen // BLOCK_SIZE))))
            drafts = self.drafter.propose(ids, [s.prompt_ids + s.output_ids for s in seqs], k,
                                          width)
        else:
            drafts = []
            for s in seqs:
                if getattr(s, "ngram", None) is None:
                    s.ngram = NGramDraft(k)
                    s.ngram.extend(s.prompt_ids + s.output_ids)
                drafts.append(s.ngram.propose(k))
        drafts = [d[:b] for d, b in zip(drafts, budget)]
        kv_lens = [s.total_len - 1 for s in seqs]
        hid = [] if self.spec == "mtp" else None
        results = verify_batch(m, ids, [s.output_ids[-1] for s in seqs], drafts, kv_lens, hid)
        if self._device_failed(seqs, out):
            return
        st = self.spec_stats
        st.rounds += 1
        metrics.SPEC_PROPOSED.labels(model=self.model_id).inc(sum(len(d) for d in drafts))
        metrics.SPEC_ACCEPTED.labels(model=self.model_id).inc(
            sum(len(r) - 1 for r in results))
        for i, (s, d, acc, kl) in enumerate(zip(seqs, drafts, results, kv_lens)):
            a = len(acc) - 1
            st.drafted += len(d)
            st.accepted += a
            st.emitted += len(acc)
            if not s.finished:
                m.kv.truncate(s.seq_id, kl + 1 + a)
                if hid is not None:
                    self.drafter.observe(s.seq_id, kl, acc, hid[i])
                if self.drafter is not None:
                    self.drafter.accept(s.seq_id, a, k)
            for t in acc:
                self._emit(s, int(t), out)
                if getattr(s, "ngram", None) is not None:
                    s.ngram.append(int(t))
                if s.finished:
                    if self.drafter is not None:
                        self.drafter.release(s.seq_id)
                    break

    # ------------------------------------------------------------ sampling
    def _pick(self, seqs: List[Sequence], logits: torch.Tensor) -> List[int]:
        m = self.model
        if all(s.task.temperature <= 0 and not self._has_penalty(s) for s in seqs):
            return [int(t) for t in m.greedy(logits).tolist()]
        return self._pick_full(seqs, m.full_logits(logits))

    def _pick_full(self, seqs: List[Sequence], full: torch.Tensor) -> List[int]:
        """Sample from full-vocabulary logits (penalties use the history)."""
        if self.dev.type != "cuda":
            outs = []
            for s, row in zip(seqs, full):
                sp = s.task.sampling
                if not hasattr(s, "_rng"):
                    s._rng = ref.init_rng(sp.seed if sp.seed is not None
                                          else self._seq_seed(s))
                outs.append(ref.sample(row, s.prompt_ids + s.output_ids, s.task.temperature,
                                       sp.top_p, sp.top_k, sp.frequency_penalty,
                                       sp.presence_penalty, 1.0, 0, s._rng))
            return outs
        B, V = full.shape
        params = torch.zeros(B, 8)
        hist_len = []
        hist = []
        seeds, offs = [], []
        for i, s in enumerate(seqs):
            sp = s.task.sampling
            params[i] = torch.tensor([s.task.temperature, sp.top_p, sp.top_k,
                                      sp.frequency_penalty, sp.presence_penalty, 1.0, 0, 0])
            h = s.prompt_ids + s.output_ids if self._has_penalty(s) else []
            hist.append(h)
            hist_len.append(len(h))
            seed = sp.seed if sp.seed is not None else self._seq_seed(s)
            seeds.append(seed)
            offs.append(s.rng_offset)
            s.rng_offset += 1
        hmax = max(1, max(hist_len))
        ht = torch.zeros(B, hmax, dtype=torch.int32)
        for i, h in enumerate(hist):
            if h:
                ht[i, :len(h)] = torch.tensor(h, dtype=torch.int32)
        work = torch.empty(B * V, dtype=torch.float32, device=self.dev)
        outt = torch.empty(B, dtype=torch.int32, device=self.dev)
        ops.sample(full.contiguous(), params.to(self.dev), ht.to(self.dev),
                   torch.tensor(hist_len, dtype=torch.int32, device=self.dev), work,
                   torch.tensor(seeds, dtype=torch.int64, device=self.dev),
                   torch.tensor(offs, dtype=torch.int64, device=self.dev), outt)
        return [int(t) for t in outt.tolist()]

    @staticmethod
    def _seq_seed(s: Sequence) -> int:
        """Sampling seed of a request without one: a stable hash of its id, so
        every replica of a tensor-parallel engine draws the same tokens."""
        import zlib

        return zlib.crc32(s.seq_id.encode()) & 0x7FFFFFFF

    def _speculable(self, s: Sequence) -> bool:
        """Greedy, unpenalised sequences without logprobs decode speculatively."""
        return s.task.temperature <= 0 and not self._has_penalty(s) and s.task.logprobs <= 0

    def _logprobs(self, rows, logits: torch.Tensor, toks) -> Dict[str, TokenLogprobs]:
        """Per-token logprobs for the rows whose task asked for them: the
        chosen token's log-probability under the model's distribution
        (log-softmax of the raw logits, before temperature and penalties) and
        the task's top-N alternatives (the OpenAI `logprobs` /
        `top_logprobs` semantics; at most 20)."""
        want = [(i, s) for i, s in rows if s.task.logprobs > 0]
        if not want:
            return {}
        full = self.model.full_logits(logits)
        idx = torch.tensor([i for i, _ in want], dtype=torch.long, device=full.device)
        lp = torch.log_softmax(full.index_select(0, idx).float(), dim=-1)
        k = max(min(20, s.task.logprobs) for _, s in want)
        top_v, top_i = lp.topk(k, dim=-1)
        chosen = torch.tensor([int(toks[i]) for i, _ in want], dtype=torch.long,
                              device=full.device)
        ch = lp.gather(1, chosen.unsqueeze(1)).squeeze(1)
        top_v, top_i, ch = top_v.cpu().tolist(), top_i.cpu().tolist(), ch.cpu().tolist()
        out = {}
        for r, (i, s) in enumerate(want):
            n = min(20, s.task.logprobs)
            tid = int(toks[i])
            out[s.seq_id] = TokenLogprobs(
                token=self.tok.decode([tid]), token_id=tid, logprob=float(ch[r]),
                top_logprobs=[TopLogprob(token=self.tok.decode([int(t)]), token_id=int(t),
                                         logprob=float(v))
                              for t, v in zip(top_i[r][:n], top_v[r][:n])])
        return out

    @staticmethod
    def _has_penalty(s: Sequence) -> bool:
        sp = s.task.sampling
        return sp.frequency_penalty != 0.0 or sp.presence_penalty != 0.0

    # ------------------------------------------------------------ emission
    def _emit(self, s: Sequence, tok: int, out, lp: Optional[TokenLogprobs] = None):
        s.output_ids.append(tok)
        if s.first_token_at is None:
            s.first_token_at = time.monotonic()
        tid = s.task.task_id
        finish = None
        if tok in self.eos:
            finish = FinishReason.STOP
        elif len(s.output_ids) >= max(1, s.task.max_tokens):
            finish = FinishReason.LENGTH
        elif s.total_len + 1 >= self.max_model_len:
            finish = FinishReason.LENGTH
        dec = self.decoders.get(tid)
        text = "" if (dec is None or tok in self.eos) else dec.push([tok])
        # n_tokens is set on every token chunk: a token whose text is still
        # an incomplete UTF-8 sequence (empty text) must still be counted.
        if finish is None:
            c = Chunk.token(tid, tok, text).with_n_tokens(1)
            c.logprobs = lp
            out.append((tid, c))
            return
        if self.drafter is not None:
            self.drafter.release(s.seq_id)
        if tok not in self.eos:
            c = Chunk.token(tid, tok, text).with_n_tokens(1)
            c.logprobs = lp
            out.append((tid, c))
        fin = Chunk.final_marker(tid, "").with_finish_reason(finish).with_prompt_tokens(
            len(s.prompt_ids)).with_cached_tokens(getattr(s, "cached_prefix", 0))
        task_done(tid, getattr(s, "submitted_at", 0.0) or 0.0, s.first_token_at or 0.0,
                  time.monotonic(), len(s.output_ids), len(s.prompt_ids))
        out.append((tid, fin))
        s.finished = True
        self.sched.remove(s.seq_id)
        self.decoders.pop(tid, None)


class LLMBuilder(Builder):
    """Builds an LLMEngine from a model preset (random init) or a shard dir."""

    def __init__(self, model: str, device: str = "cuda", kv_blocks: int = 0,
                 kv_fraction: float = 0.5, max_running: int = 64, max_model_len: int = 8192,
                 prefix_cache_blocks: int = 0, use_graph: bool = True, seed: int = 0,
                 tp=None, tokenizer_path: Optional[str] = None, spec: Optional[str] = None,
                 spec_k: int = 4, draft_model: Optional[str] = None, draft_kv_blocks: int = 0,
                 ep=None, max_prefill_tokens: int = 8192):
        self.ep = ep  # parallel.ep.ExpertParallel: this rank's share of the experts
        self.max_prefill_tokens = max_prefill_tokens
        self.spec = spec
        self.spec_k = spec_k
        self.draft_name = draft_model
        self.draft_kv_blocks = draft_kv_blocks
        self.draft = None
        self.mtp = None
        self.model_name = model
        self.device = device
        self.kv_blocks = kv_blocks
        self.kv_fraction = kv_fraction
        self.max_running = max_running
        self.max_model_len = max_model_len
        self.prefix_cache_blocks = prefix_cache_blocks
        self.use_graph = use_graph
        self.seed = seed
        self.tp = tp
        self.tokenizer_path = tokenizer_path
        self.model = None
        self.tokenizer = None

    def connect(self, peers: PeerLayout) -> None:
        pass

    def model_class(self, cfg):
        """Dense Llama-family model, or the sparse-MoE model for MoE configs
        (hybrid Gated-DeltaNet MoE, MLA MoE, plain MoE)."""
        if cfg.is_gemma4:
            from ..models.gemma4 import Gemma4Model

            return Gemma4Model
        if cfg.is_hybrid:
            from ..models.qwen36 import HybridMoEModel

            return HybridMoEModel
        if cfg.is_dsa:
            from ..models.glm5 import GLM5Model

            return GLM5Model
        if cfg.is_mla:
            from ..models.mla import MLAModel

            return MLAModel
        if cfg.is_moe:
            from ..models.moe import MoEModel

            return MoEModel
        from ..models.llama import LlamaModel

        return LlamaModel

    def load(self, shard: ShardSpec) -> Iterable[LoadProgress]:
        import os

        from ..api.templates import load_tokenizer
        from ..models.config import get_config

        yield LoadProgress.msg(f"loading {self.model_name}")
        if os.path.isdir(self.model_name) and os.path.exists(
                os.path.join(self.model_name, "manifest.json")):
            from ..shard.moe_format import load_moe_model

            self.model = load_moe_model(self.model_name, self.device)
            tok_dir = self.tokenizer_path
        elif os.path.isdir(self.model_name):
            from ..shard.format import load_stage_model

            self.model = load_stage_model(self.model_name, shard, self.device, tp=self.tp)
            tok_dir = self.tokenizer_path or os.path.join(os.path.dirname(
                os.path.abspath(self.model_name.rstrip("/"))), "tokenizer")
            if not os.path.isdir(tok_dir):
                tok_dir = os.path.join(self.model_name, "tokenizer")
        else:
            cfg = get_config(self.model_name)
            extra = {"ep": self.ep} if self.ep is not None else {}
            self.model = self.model_class(cfg)(cfg, self.device, tp=self.tp,
                                               layer_start=shard.layer_start,
                                               layer_end=shard.layer_end,
                                               has_embed=shard.is_first_stage,
                                               has_head=shard.is_last_stage,
                                               **extra).init_random(seed=self.seed)
            tok_dir = self.tokenizer_path
        cfg = self.model.cfg
        self.tokenizer = load_tokenizer(tok_dir, cfg.vocab_size, cfg.eos_token_ids[0])
        blocks = self.kv_blocks
        hybrid = cfg.is_hybrid
        if hybrid and (self.spec or self.prefix_cache_blocks):
            raise InvalidConfig("the linear-attention state of this model cannot be shared or "
                                "rewound: no prefix cache, no speculative decoding")
        if blocks <= 0:
            per = self.model.kv_bytes_per_block()
            if torch.device(self.device).type == "cuda":
                free, _ = torch.cuda.mem_get_info(torch.device(self.device))
                if hybrid:  # recurrent state of every running sequence first
                    free -= self.max_running * self.model.state_bytes_per_seq()
                blocks = max(64, int(free * self.kv_fraction) // per)
            else:
                blocks = max(64, (self.max_running * self.max_model_len) // BLOCK_SIZE // 4)
        tp = self.tp
        if tp is not None and tp.size > 1:
            # Replicated schedulers must see the same pool: the smallest
            # rank's block count wins.
            t = torch.tensor([blocks], dtype=torch.int64,
                             device=self.device if torch.device(self.device).type == "cuda"
                             else "cpu")
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MIN, group=tp.group)
            blocks = int(t.item())
        if hybrid:
            self.model.allocate_kv(blocks, max_seqs=self.max_running)
        else:
            self.model.allocate_kv(blocks)
        yield LoadProgress.msg(f"kv cache: {blocks} blocks")
        if self.spec == "draft":
            if not self.draft_name:
                raise InvalidConfig("--spec draft needs --draft-model")
            from ..models.llama import LlamaModel

            dcfg = get_config(self.draft_name)
            if dcfg.vocab_size != cfg.vocab_size:
                raise InvalidConfig("draft and target vocabularies differ")
            self.draft = LlamaModel(dcfg, self.device).init_random(seed=self.seed + 1)
            self.draft.allocate_kv(self.draft_kv_blocks or blocks)
            yield LoadProgress.msg(f"draft model {self.draft_name} loaded")
        if self.spec == "mtp":
            if not cfg.num_nextn_predict_layers or not cfg.is_dsa:
                raise InvalidConfig("--spec mtp needs a GLM-5 model with an MTP layer")
            if self.prefix_cache_blocks:
                raise InvalidConfig("--spec mtp does not combine with the prefix cache")
            from ..models.glm5 import GLM5MTP

            self.mtp = GLM5MTP(self.model).init_random(seed=self.seed + 2)
            self.mtp.allocate_kv(blocks)
            yield LoadProgress.msg("MTP draft head loaded")
        yield LoadProgress.done()

    def build(self) -> Engine:
        if self.model is None:
            raise NotLoaded()
        return LLMEngine(self.model, self.tokenizer, max_running=self.max_running,
                         max_prefill_tokens=self.max_prefill_tokens,
                         max_model_len=self.max_model_len, use_graph=self.use_graph,
                         prefix_cache_blocks=self.prefix_cache_blocks,
                         model_id=self.model_name, spec=self.spec, draft_model=self.draft,
                         spec_k=self.spec_k, mtp_head=self.mtp)


class MoEBuilder(LLMBuilder):
    """Builder of the sparse-MoE engine (Qwen3-MoE / Kimi-K2 / GLM-5 / Qwen3.6
    shapes).  The counterpart of the reference's sparse-MoE engines
    (crates/cascadia-engine-sparse-moe/src/engine.rs, glm/model.rs): the same
    continuous-batching LLMEngine drives the routed-expert model (fused
    router/top-k kernel, counting-sort permute, grouped INT4 expert GEMMs,
    weighted combine); dense presets are rejected."""

    def model_class(self, cfg):
        if not cfg.is_moe:
            raise InvalidConfig(f"{self.model_name}: not a sparse-MoE config")
        return super().model_class(cfg)
