"""Paged KV cache storage (block size 16) and its block allocator.

Replaces the reference's per-engine KV handling (OpenVINO stateful KV, the
host-side ring ``StaticKv`` in crates/cascadia-engine-openvino/src/runtime.rs:1067-1236
and the geometric-grow bf16 buffers of crates/cascadia-engine-sparse-moe/src/runner.rs:2788-2960)
with one device pool addressed through per-sequence block tables.

Storage layout: ``[num_layers, num_blocks, kv_heads, 16, head_dim]`` for K and
for V, so that one (layer, block, head) tile is contiguous for TMA.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional

import torch

BLOCK_SIZE = 16


class BlockAllocator:
    """Free-list allocator with reference counts (for prefix sharing)."""

    def __init__(self, num_blocks: int):
        self.num_blocks = num_blocks
        self._free: List[int] = list(range(num_blocks - 1, -1, -1))
        self._ref = [0] * num_blocks

    @property
    def num_free(self) -> int:
        return len(self._free)

    def allocate(self, n: int) -> List[int]:
        if n > len(self._free):
            raise MemoryError(f"KV cache exhausted: need {n} blocks, {len(self._free)} free")
        out = [self._free.pop() for _ in range(n)]
        for b in out:
            self._ref[b] = 1
        return out

    def incref(self, blocks: List[int]):
        for b in blocks:
            self._ref[b] += 1

    def free(self, blocks: List[int]):
        for b in blocks:
            self._ref[b] -= 1
            if self._ref[b] == 0:
                self._free.append(b)
            elif self._ref[b] < 0:
                raise RuntimeError(f"double free of KV block {b}")

    def refcount(self, b: int) -> int:
        return self._ref[b]


@dataclass
class SeqKV:
    """Block table and length of one sequence."""
    blocks: List[int] = field(default_factory=list)
    length: int = 0

    def slots(self, start: int, end: int) -> List[int]:
        return [self.blocks[p // BLOCK_SIZE] * BLOCK_SIZE + p % BLOCK_SIZE
                for p in range(start, end)]


class KVCache:
    """Device K/V pools for the layers held by this rank."""

    def __init__(self, num_layers: int, num_blocks: int, kv_heads: int, head_dim: int,
                 device, dtype=torch.bfloat16, v_head_dim: Optional[int] = None):
        self.num_layers = num_layers
        self.num_blocks = num_blocks
        self.kv_heads = kv_heads
        self.head_dim = head_dim
        shape = (num_layers, num_blocks, kv_heads, BLOCK_SIZE, head_dim)
        # Zero-init: kernels read whole 16-token blocks, so never-written
        # slots must hold finite values.
        self.k = torch.zeros(shape, dtype=dtype, device=device)
        vshape = (num_layers, num_blocks, kv_heads, BLOCK_SIZE, v_head_dim or head_dim)
        self.v = torch.zeros(vshape, dtype=dtype, device=device)
        self.allocator = BlockAllocator(num_blocks)
        self.seqs: Dict[str, SeqKV] = {}

    @staticmethod
    def bytes_per_block(num_layers, kv_heads, head_dim, dtype_bytes=2) -> int:
        return 2 * num_layers * kv_heads * BLOCK_SIZE * head_dim * dtype_bytes

    # ------------------------------------------------------------ sequences
    def add_sequence(self, seq_id: str, shared_prefix: Optional[List[int]] = None) -> SeqKV:
        s = SeqKV()
        if shared_prefix:
            self.allocator.incref(shared_prefix)
            s.blocks = list(shared_prefix)
            s.length = len(shared_prefix) * BLOCK_SIZE
        self.seqs[seq_id] = s
        return s

    def reserve(self, seq_id: str, new_length: int):
        """Grow the block table so that `new_length` tokens fit."""
        s = self.seqs[seq_id]
        need = (new_length + BLOCK_SIZE - 1) // BLOCK_SIZE - len(s.blocks)
        if need > 0:
            s.blocks.extend(self.allocator.allocate(need))

    def can_reserve(self, seq_id: Optional[str], new_length: int) -> bool:
        have = len(self.seqs[seq_id].blocks) if seq_id in self.seqs else 0
        need = (new_length + BLOCK_SIZE - 1) // BLOCK_SIZE - have
        return need <= self.allocator.num_free

    def truncate(self, seq_id: str, new_length: int):
        """Rewind (speculative decoding): drop tokens past `new_length`."""
        s = self.seqs[seq_id]
        s.length = min(s.length, new_length)
        keep = (s.length + BLOCK_SIZE - 1) // BLOCK_SIZE
        if keep < len(s.blocks):
            self.allocator.free([b for b in s.blocks[keep:] if b >= 0])
            s.blocks = s.blocks[:keep]

    def evict_before(self, seq_id: str, first_needed: int, sinks: int = 0) -> int:
        """Sliding-window attention: return the blocks whose positions all lie
        before ``first_needed`` (and past the ``sinks`` first positions) to
        the pool.  Their table entries become -1 (the kernels never read
        them; the device tables carry block 0 there).  Returns blocks freed."""
        s = self.seqs[seq_id]
        lo = -(-sinks // BLOCK_SIZE)
        hi = min(len(s.blocks), max(0, first_needed) // BLOCK_SIZE)
        gone = [j for j in range(lo, hi) if s.blocks[j] >= 0]
        if gone:
            self.allocator.free([s.blocks[j] for j in gone])
            for j in gone:
                s.blocks[j] = -1
        return len(gone)

    def slide(self, seq_id: str, cfg, first_query_pos: int):
        """Free what a sliding-window model no longer reads (no-op without
        a window): blocks wholly before the earliest key the queries from
        ``first_query_pos`` on can see."""
        w = getattr(cfg, "sliding_window", 0)
        if w > 0:
            self.evict_before(seq_id, first_query_pos - w + 1, cfg.attention_sinks)

    def free_sequence(self, seq_id: str):
        s = self.seqs.pop(seq_id, None)
        if s is not None:
            self.allocator.free([b for b in s.blocks if b >= 0])

    def block_table(self, seq_ids: List[str], width: int, device) -> torch.Tensor:
        t = torch.zeros(len(seq_ids), width, dtype=torch.int32)
        for i, sid in enumerate(seq_ids):
            b = self.seqs[sid].blocks
            t[i, :len(b)] = torch.tensor(b, dtype=torch.int32).clamp_min(0)
        return t.to(device, non_blocking=True)

    def gather(self, layer: int, seq_id: str):
        """Dense [len, H, D] copies of one sequence's K/V (CPU oracle path)."""
        s = self.seqs[seq_id]
        ids = torch.tensor(s.blocks, dtype=torch.long, device=self.k.device).clamp_min(0)
        k = self.k[layer, ids].permute(0, 2, 1, 3).reshape(-1, self.kv_heads, self.k.shape[-1])
        v = self.v[layer, ids].permute(0, 2, 1, 3).reshape(-1, self.kv_heads, self.v.shape[-1])
        return k, v
