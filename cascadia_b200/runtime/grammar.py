"""Grammar-constrained decoding with forced-run batching.

Where a grammar (a JSON or tool-call schema, a template) admits exactly one
continuation, those tokens are emitted without a model forward of their own:
the whole forced run is appended to the KV cache in ONE multi-token forward
(the prefill path, mid-stream), whose last row gives the distribution at the
next free position.  At a free position the logits are masked to the tokens
the grammar allows before the argmax.  K forced tokens cost one forward
instead of K.  (The reference's GLM-5 shell has the same contract:
crates/cascadia-engine-sparse-moe/src/glm/grammar.rs:1-60 ``Grammar``,
``masked_argmax``, ``GrammarOutput``.)
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Protocol, Sequence

import torch

from ..models.llama import build_batch


class Grammar(Protocol):
    def forced_run(self, emitted: Sequence[int]) -> List[int]:
        """The maximal run of tokens the grammar forces next (empty when the
        next token is a free choice)."""

    def allowed(self, emitted: Sequence[int], vocab: int) -> Optional[torch.Tensor]:
        """Bool mask [vocab] of the tokens legal at a free position (None:
        every token)."""

    def can_end(self, emitted: Sequence[int]) -> bool:
        """Whether generation may stop after ``emitted``."""


@dataclass
class GrammarOutput:
    tokens: List[int]
    forwards: int           # model forwards spent (< len(tokens) when runs were forced)


def masked_argmax(logits: torch.Tensor, mask: Optional[torch.Tensor]) -> int:
    """Index of the largest allowed logit (lowest index on ties)."""
    x = logits.float().reshape(-1)
    if mask is not None:
        x = x.masked_fill(~mask.to(x.device), float("-inf"))
        if not bool(torch.isfinite(x).any()):
            raise ValueError("grammar allows no token at a free position")
    return int(torch.argmax(x))


class TemplateGrammar:
    """A token template: fixed tokens are forced, ``None`` marks a free slot
    whose token must come from ``choices`` (or any token when empty).  The
    grammar accepts once every slot is filled."""

    def __init__(self, template: Sequence[Optional[int]], choices: Sequence[int] = ()):
        self.template = list(template)
        self.choices = list(choices)

    def forced_run(self, emitted):
        run = []
        i = len(emitted)
        while i < len(self.template) and self.template[i] is not None:
            run.append(self.template[i])
            i += 1
        return run

    def allowed(self, emitted, vocab):
        if not self.choices:
            return None
        m = torch.zeros(vocab, dtype=torch.bool)
        m[torch.tensor(self.choices)] = True
        return m

    def can_end(self, emitted):
        return len(emitted) >= len(self.template)


def generate_constrained(model, seq_id: str, prompt: Sequence[int], grammar: Grammar,
                         max_tokens: int, eos: Sequence[int] = ()) -> GrammarOutput:
    """Greedy generation of one sequence under ``grammar`` with forced runs
    batched into single forwards.  The sequence's KV is freed at the end."""
    m = model
    dev = m.device
    V = m.cfg.vocab_size
    kv = m.kv
    kv.add_sequence(seq_id)

    def feed(tokens: List[int], start: int) -> torch.Tensor:
        batch = build_batch(m, [seq_id], [len(tokens)], [start], len(tokens) == 1)
        hid = m.embed_tokens(torch.tensor(tokens, dtype=torch.int32, device=dev))
        m.forward(batch, hid)
        return m.head(hid[-1:].contiguous())[0]

    out: List[int] = []
    forwards = 0
    try:
        logits = feed(list(prompt), 0)
        forwards += 1
        fed = len(prompt)                 # tokens with KV written
        pending: Optional[int] = None     # emitted, not fed yet
        while len(out) < max_tokens:
            run = grammar.forced_run(out)[:max_tokens - len(out)]
            if run:
                out.extend(run)
                rows = ([pending] if pending is not None else []) + run
                logits = feed(rows, fed)
                forwards += 1
                fed += len(rows)
                pending = None
                continue
            if grammar.can_end(out):
                break
            if pending is not None:
                logits = feed([pending], fed)
                forwards += 1
                fed += 1
            t = masked_argmax(logits, grammar.allowed(out, V))
            out.append(t)
            pending = t
            if t in eos or grammar.can_end(out):
                break
    finally:
        kv.free_sequence(seq_id)
    return GrammarOutput(out, forwards)
