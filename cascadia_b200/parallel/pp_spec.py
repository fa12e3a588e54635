"""Distributed speculative decoding across pipeline stages.

The reference's ``ov-dist-spec`` engine keeps the draft model and target
stage 0 on the driver rank and the later target stages on the workers; one
round drafts ``k`` tokens greedily, verifies ``[pending, d1 .. dk]`` in one
multi-token forward through the target pipeline and keeps the longest
accepted prefix plus the correction token, rewinding the KV by mask
(crates/cascadia-engine-openvino/src/dist_spec.rs:958-1128
``spec_decode_greedy``, frames :48-65).

Here every rank runs :class:`PipelinedSpecDecoder` in lockstep over
``torch.distributed`` (NCCL on GPUs, gloo on CPUs):

1. rank 0 drafts for the live sequences (a draft model on its GPU, or
   n-gram prompt lookup) and broadcasts the rows to verify;
2. the rows go through the stages as one ragged multi-token batch (hidden
   rows by point-to-point send/recv, exactly like the pipelined prefill);
3. the last stage takes the argmax of every row and runs the verify
   (longest accepted prefix + correction token), then broadcasts the
   accepted tokens to every rank;
4. every stage resets its paged KV length to the accepted prefix (blocks
   past it return to the pool).  The output equals plain greedy decoding of
   the target.
"""
from __future__ import annotations

from typing import List, Optional, Sequence

import torch
import torch.distributed as dist

from ..models.llama import build_batch
from ..runtime.kv_cache import BLOCK_SIZE
from ..runtime.spec import ModelDrafter, NGramDraft, SpecStats
from .pp_decode import pp_prefill


class PipelinedSpecDecoder:
    def __init__(self, model, stage: int, n_stages: int, k: int = 4, draft=None,
                 group=None, ranks: Optional[Sequence[int]] = None, use_graph: bool = True):
        self.m = model
        self.stage, self.S = stage, n_stages
        self.ranks = list(ranks) if ranks is not None else list(range(n_stages))
        self.group = group
        # Every rank must agree on k (it sizes the control tensors).
        self.k = k
        self.drafter = ModelDrafter(draft, use_graph) if (draft is not None and stage == 0) else None
        self.use_ngram = draft is None
        self.stats = SpecStats()
        dev = model.device
        # Collectives of the control plane run on the device NCCL uses.
        self.cdev = dev if dist.get_backend(group) == "nccl" else torch.device("cpu")

    # ------------------------------------------------------------ plumbing
    def _bcast(self, t: torch.Tensor, src_stage: int) -> torch.Tensor:
        t = t.to(self.cdev)
        dist.broadcast(t, self.ranks[src_stage], group=self.group)
        return t.cpu()

    def _forward_rows(self, seq_ids, lens, kv_lens, flat_tokens):
        """Rows through this stage; returns the argmax of every row on the
        last stage (None elsewhere)."""
        m = self.m
        batch = build_batch(m, seq_ids, lens, kv_lens, False)
        T = sum(lens)
        if self.stage == 0:
            hidden = m.embed_tokens(torch.tensor(flat_tokens, dtype=torch.int32, device=m.device))
        else:
            hidden = torch.empty(T, m.cfg.hidden_size, dtype=torch.bfloat16, device=m.device)
            dist.recv(hidden, self.ranks[self.stage - 1], group=self.group)
        m.forward(batch, hidden)
        if self.stage < self.S - 1:
            dist.send(hidden, self.ranks[self.stage + 1], group=self.group)
            return None
        return m.greedy(m.head(hidden)).to(torch.int32).cpu()

    # ------------------------------------------------------------ generate
    def generate(self, prompts: Sequence[Sequence[int]], max_new_tokens: int,
                 eos: Sequence[int] = (), prefix: str = "ds") -> List[List[int]]:
        """Every rank calls this with the same prompts; returns the generated
        tokens (the same lists on every rank)."""
        from ..ops import reference as ref

        m = self.m
        n = len(prompts)
        ids = [f"{prefix}{i}" for i in range(n)]
        longest = max(len(p) for p in prompts) + max_new_tokens + self.k + 2
        width = -(-longest // BLOCK_SIZE)
        first = pp_prefill(m, self.stage, self.S, ids, [list(p) for p in prompts], self.group,
                           self.ranks)
        firsts = self._bcast(torch.tensor(first if self.stage == 0 else [0] * n,
                                          dtype=torch.int64), 0).tolist()
        tokens = [list(p) + [int(t)] for p, t in zip(prompts, firsts)]
        kv_len = [len(p) for p in prompts]
        generated = [1] * n
        done = [max_new_tokens <= 1 or t in eos for t in firsts]
        ngrams = None
        if self.stage == 0 and self.use_ngram:
            ngrams = []
            for tk in tokens:
                g = NGramDraft(self.k)
                g.extend(tk)
                ngrams.append(g)
        K = self.k
        while True:
            live = [i for i in range(n) if not done[i]]
            if not live:
                break
            # 1. drafts on rank 0; every rank receives the rows
            #    [pending, d1 .. dk] (col 0: row length, -1 padding).
            ctrl = torch.full((n, K + 2), -1, dtype=torch.int64)
            if self.stage == 0:
                if self.drafter is not None:
                    drafts = self.drafter.propose([ids[i] for i in live],
                                                  [tokens[i] for i in live], K, width)
                else:
                    drafts = [ngrams[i].propose(K) for i in live]
                for j, i in enumerate(live):
                    d = drafts[j][:max(0, max_new_tokens - generated[i] - 1)][:K]
                    row = [tokens[i][-1]] + d
                    ctrl[j, 0] = len(row)
                    ctrl[j, 1:1 + len(row)] = torch.tensor(row)
            ctrl = self._bcast(ctrl, 0)
            lens = [int(ctrl[j, 0]) for j in range(len(live))]
            rows = [ctrl[j, 1:1 + lens[j]].tolist() for j in range(len(live))]
            # 2. verify forward through the stages.
            picks = self._forward_rows([ids[i] for i in live], lens, [kv_len[i] for i in live],
                                       [t for r in rows for t in r])
            # 3. the last stage keeps the longest accepted prefix + the
            #    correction token of each row and tells everyone.
            res = torch.full((n, K + 1), -1, dtype=torch.int64)
            if self.stage == self.S - 1:
                off = 0
                for j in range(len(live)):
                    tgt = picks[off:off + lens[j]].tolist()
                    acc = ref.spec_verify(tgt, rows[j][1:])
                    res[j, :len(acc)] = torch.tensor(acc)
                    off += lens[j]
            res = self._bcast(res, self.S - 1)
            # 4. identical bookkeeping on every rank.
            for j, i in enumerate(live):
                acc = [int(t) for t in res[j].tolist() if t >= 0]
                a = len(acc) - 1
                self.stats.drafted += lens[j] - 1
                self.stats.accepted += a
                new = acc[:max_new_tokens - generated[i]]
                for q, t in enumerate(new):
                    if t in eos:
                        new = new[:q + 1]
                        break
                kv_len[i] += 1 + a
                m.kv.truncate(ids[i], kv_len[i])
                if self.drafter is not None:
                    self.drafter.accept(ids[i], a, K)
                tokens[i].extend(new)
                if ngrams is not None:
                    ngrams[i].extend(new)
                generated[i] += len(new)
                self.stats.emitted += len(new)
                if generated[i] >= max_new_tokens or (new and new[-1] in eos):
                    done[i] = True
            self.stats.rounds += 1
        for sid in ids:
            m.kv.free_sequence(sid)
            if self.drafter is not None:
                self.drafter.release(sid)
        return [tokens[i][len(prompts[i]):] for i in range(n)]
