"""Continuous-batching scheduler state and the paged-KV prefix cache.

Replaces the reference's single-request engine mutex and its packed
multi-slot "seq-as-batch" scheme (crates/cascadia-engine-openvino/src/packed.rs:1-24,
PackedKv :97-330) with real batching: every engine iteration runs one
prefill chunk (bounded by ``max_prefill_tokens``) and one decode step of all
running sequences.  Prefix sharing (the reference's KV prefix cache,
crates/cascadia-engine-sparse-moe/src/kv_prefix_cache.rs:172-335, keyed by a
prefix hash + model fingerprint) becomes block-level sharing: full 16-token
blocks are hashed as a chain and reused by reference count.
"""
from __future__ import annotations

import collections
import hashlib
import time
from dataclasses import dataclass, field
from typing import Deque, Dict, List, Optional, Tuple

from ..types import GenerationTask
from .kv_cache import BLOCK_SIZE, KVCache


@dataclass
class Sequence:
    task: GenerationTask
    prompt_ids: List[int]
    seq_id: str
    output_ids: List[int] = field(default_factory=list)
    prefilled: int = 0          # prompt tokens already in the KV cache
    emitted_text: str = ""
    rng_offset: int = 0
    arrived: float = field(default_factory=time.monotonic)
    first_token_at: Optional[float] = None
    finished: bool = False
    cached_prefix: int = 0      # prompt tokens served from the prefix cache

    @property
    def total_len(self) -> int:
        return len(self.prompt_ids) + len(self.output_ids)

    @property
    def in_prefill(self) -> bool:
        return self.prefilled < len(self.prompt_ids)


class PrefixCache:
    """Hash-chained full blocks -> block id, refcounted through the allocator.

    A cached block stays allocated (refcount >= 1 held by the cache) until it
    is evicted (LRU) to make room.
    """

    def __init__(self, kv: KVCache, fingerprint: str, max_blocks: int):
        self.kv = kv
        self.fp = fingerprint
        self.max_blocks = max_blocks
        self.map: "collections.OrderedDict[str, int]" = collections.OrderedDict()

    def _hashes(self, ids: List[int], n_blocks: int) -> List[str]:
        out, h = [], hashlib.sha1(self.fp.encode())
        for b in range(n_blocks):
            h = h.copy()
            h.update(bytes(str(ids[b * BLOCK_SIZE:(b + 1) * BLOCK_SIZE]), "ascii"))
            out.append(h.hexdigest())
        return out

    def lookup(self, ids: List[int]) -> List[int]:
        """Longest cached run of full blocks for this prompt (leave >= 1 token
        to compute so the last position's logits exist)."""
        n = (len(ids) - 1) // BLOCK_SIZE
        blocks = []
        for h in self._hashes(ids, n):
            b = self.map.get(h)
            if b is None:
                break
            self.map.move_to_end(h)
            blocks.append(b)
        return blocks

    def insert(self, ids: List[int], blocks: List[int], n_tokens: int):
        n = min(n_tokens // BLOCK_SIZE, len(blocks))
        for h, b in zip(self._hashes(ids, n), blocks[:n]):
            if h in self.map:
                continue
            self.kv.allocator.incref([b])
            self.map[h] = b
        while len(self.map) > self.max_blocks:
            self.evict_one()

    def evict_one(self) -> bool:
        if not self.map:
            return False
        _, b = self.map.popitem(last=False)
        self.kv.allocator.free([b])
        return True

    def clear(self):
        while self.evict_one():
            pass


class SchedulerState:
    def __init__(self, kv: KVCache, max_running: int, max_prefill_tokens: int,
                 prefix_cache: Optional[PrefixCache] = None, max_queue: int = 1024):
        self.kv = kv
        self.max_running = max_running
        self.max_prefill_tokens = max_prefill_tokens
        self.prefix = prefix_cache
        self.max_queue = max_queue
        self.waiting: Deque[Sequence] = collections.deque()
        self.running: List[Sequence] = []
        self.by_id: Dict[str, Sequence] = {}

    def add(self, seq: Sequence):
        self.waiting.append(seq)
        self.by_id[seq.seq_id] = seq

    def remove(self, seq_id: str) -> Optional[Sequence]:
        s = self.by_id.pop(seq_id, None)
        if s is None:
            return None
        if s in self.running:
            self.running.remove(s)
        else:
            try:
                self.waiting.remove(s)
            except ValueError:
                pass
        if seq_id in self.kv.seqs:
            if self.prefix is not None and not s.in_prefill:
                self.prefix.insert(s.prompt_ids, self.kv.seqs[seq_id].blocks, s.prefilled)
            self.kv.free_sequence(seq_id)
        return s

    def _blocks_needed(self, n_tokens: int) -> int:
        return (n_tokens + BLOCK_SIZE - 1) // BLOCK_SIZE

    def admit(self) -> List[Tuple[Sequence, int, int]]:
        """Pick prefill work: list of (seq, start, n_tokens) within budget."""
        work = []
        budget = self.max_prefill_tokens
        # Continue sequences already in chunked prefill first.
        for s in self.running:
            if s.in_prefill and budget > 0:
                n = min(budget, len(s.prompt_ids) - s.prefilled)
                if not self.kv.can_reserve(s.seq_id, s.prefilled + n):
                    break
                work.append((s, s.prefilled, n))
                budget -= n
        while self.waiting and budget > 0 and len(self.running) < self.max_running:
            s = self.waiting[0]
            if s.seq_id not in self.kv.seqs:
                shared = self.prefix.lookup(s.prompt_ids) if self.prefix else []
                need = self._blocks_needed(len(s.prompt_ids) + 1) - len(shared)
                while need > self.kv.allocator.num_free and self.prefix and self.prefix.evict_one():
                    pass
                if need > self.kv.allocator.num_free:
                    break  # wait for memory
                self.kv.add_sequence(s.seq_id, shared_prefix=shared)
                s.prefilled = len(shared) * BLOCK_SIZE
                s.cached_prefix = s.prefilled
            n = min(budget, len(s.prompt_ids) - s.prefilled)
            self.waiting.popleft()
            self.running.append(s)
            work.append((s, s.prefilled, n))
            budget -= n
        return work

    def decode_set(self) -> List[Sequence]:
        return [s for s in self.running if not s.in_prefill and not s.finished]
