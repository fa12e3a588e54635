"""Symmetric INT4 group quantisation and the kernel weight layout.

Canonical (checkpoint) form, shared by both reference formats:

* packed: int32 ``[N, K/8]``; word ``i`` holds columns ``8i..8i+7``, column
  ``8i+j`` in bits ``4j..4j+3`` (little-endian nibbles, even column low), as in
  crates/cascadia-int4-gemm/src/lib.rs:11-22.
* scales: ``[N, K/G]``; value = ``(nibble - 8) * scale``.
  F2 (``cascadia shard`` dense layers): G = 128, fp16 scales
  (tools/export_shards.py:1432-1438).  F1 (experts): G = 32, bf16 scales
  (crates/cascadia-int4-gemm/src/kernel.rs:46-70).

Kernel ("blob") form, produced once at load time by :func:`pack_blob`: for
every (128-row tile, 128-wide k-block) an 8 KiB block of packed rows (64 bytes
per row, nibble order within each 32-bit word ``c0,c2,c4,c6`` in the low
half-words and ``c1,c3,c5,c7`` in the high ones so that one shift+mask yields a
bf16x2 pair; the four 16-byte chunks of row ``r`` XOR-swizzled by
``(r >> 1) & 3``) followed by that block's bf16 scales.  The GEMM kernel fetches
one such block with a single bulk TMA copy.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch


@dataclass
class Int4Weight:
    packed: torch.Tensor  # int32 [N, K/8]
    scales: torch.Tensor  # fp16/bf16 [N, K/G]
    group_size: int = 128

    @property
    def n(self) -> int:
        return self.packed.shape[0]

    @property
    def k(self) -> int:
        return self.packed.shape[1] * 8

    # -------------------------------------------------------------- creation
    @staticmethod
    def quantize(w: torch.Tensor, group_size: int = 128,
                 scale_dtype: torch.dtype = torch.float16) -> "Int4Weight":
        """Symmetric per-group INT4 of a float matrix [N, K].

        Scales are rounded to bf16 first so that they are exact in both fp16
        (the F2 on-disk dtype) and bf16 (what the kernel multiplies with).
        """
        n, k = w.shape
        assert k % group_size == 0 and k % 8 == 0
        wf = w.float().view(n, k // group_size, group_size)
        amax = wf.abs().amax(-1).clamp_min(1e-8)
        scale = (amax / 7.0).to(torch.bfloat16).float()
        q = torch.clamp(torch.round(wf / scale.unsqueeze(-1)), -8, 7) + 8
        q = q.view(n, k).to(torch.int32)
        return Int4Weight(pack_nibbles(q), scale.to(scale_dtype), group_size)

    @staticmethod
    def random(n: int, k: int, std: float = 0.02, group_size: int = 128,
               generator: Optional[torch.Generator] = None, device="cpu",
               scale_dtype: torch.dtype = torch.float16) -> "Int4Weight":
        w = torch.randn(n, k, generator=generator, device=device) * std
        return Int4Weight.quantize(w, group_size, scale_dtype)

    # -------------------------------------------------------------- views
    def unpack(self) -> torch.Tensor:
        """uint8-valued int32 [N, K] nibbles (0..15)."""
        return unpack_nibbles(self.packed)

    def dequant_bf16(self) -> torch.Tensor:
        q = self.unpack().float() - 8.0
        s = self.scales.to(torch.bfloat16).float()
        s = s.repeat_interleave(self.group_size, dim=1)
        return (q * s).to(torch.bfloat16)

    def rows(self, start: int, end: int) -> "Int4Weight":
        return Int4Weight(self.packed[start:end].contiguous(), self.scales[start:end].contiguous(),
                          self.group_size)

    def cols(self, start: int, end: int) -> "Int4Weight":
        assert start % self.group_size == 0 and end % self.group_size == 0
        return Int4Weight(self.packed[:, start // 8:end // 8].contiguous(),
                          self.scales[:, start // self.group_size:end // self.group_size].contiguous(),
                          self.group_size)

    @staticmethod
    def cat_rows(ws) -> "Int4Weight":
        g = ws[0].group_size
        return Int4Weight(torch.cat([w.packed for w in ws]), torch.cat([w.scales for w in ws]), g)

    def to(self, device) -> "Int4Weight":
        return Int4Weight(self.packed.to(device), self.scales.to(device), self.group_size)

    def blob(self, interleave_gate_up: bool = False) -> torch.Tensor:
        return pack_blob(self.unpack(), self.scales, self.group_size, interleave_gate_up)


def pack_nibbles(q: torch.Tensor) -> torch.Tensor:
    """int [N, K] values 0..15 -> int32 [N, K/8] (column 8i+j at bits 4j)."""
    n, k = q.shape
    q = q.to(torch.int64).view(n, k // 8, 8)
    shifts = torch.arange(0, 32, 4, device=q.device, dtype=torch.int64)
    words = (q << shifts).sum(-1)
    words = torch.where(words >= 2**31, words - 2**32, words)
    return words.to(torch.int32)


def unpack_nibbles(packed: torch.Tensor) -> torch.Tensor:
    n, kw = packed.shape
    w = packed.to(torch.int64) & 0xFFFFFFFF
    shifts = torch.arange(0, 32, 4, device=packed.device, dtype=torch.int64)
    q = (w.unsqueeze(-1) >> shifts) & 0xF
    return q.view(n, kw * 8).to(torch.int32)


def interleave_rows(x: torch.Tensor) -> torch.Tensor:
    """[2I, ...] = [gate; up] -> rows alternate gate_j, up_j.

    Every 128-row tile then holds 64 (gate, up) pairs in adjacent rows, i.e.
    adjacent TMEM lanes, so the GEMM epilogue forms SiLU(gate) * up with one
    lane shuffle."""
    two_i = x.shape[0]
    i = two_i // 2
    assert i % 64 == 0, "intermediate size must be a multiple of 64"
    return torch.stack([x[:i], x[i:]], dim=1).reshape(two_i, *x.shape[1:])


def pack_blob(q: torch.Tensor, scales: torch.Tensor, group_size: int,
              interleave_gate_up: bool = False) -> torch.Tensor:
    """Build the kernel weight blob (uint8, 1-D) from nibbles [N, K] + scales."""
    n, k = q.shape
    assert n % 128 == 0 and k % 128 == 0, "N and K must be multiples of 128"
    sc = scales.to(torch.bfloat16)
    if interleave_gate_up:
        q = interleave_rows(q)
        sc = interleave_rows(sc)
    rt, kb = n // 128, k // 128
    qt = q.to(torch.int64).view(rt, 128, kb, 128).permute(0, 2, 1, 3).reshape(rt, kb, 128, 16, 8)
    word = torch.zeros(rt, kb, 128, 16, dtype=torch.int64, device=q.device)
    for h in range(4):
        word |= qt[..., 2 * h] << (4 * h)
        word |= qt[..., 2 * h + 1] << (16 + 4 * h)
    word = torch.where(word >= 2**31, word - 2**32, word).to(torch.int32)
    # Swizzle the four 16-byte chunks of each 64-byte row: chunk c of row r is
    # stored at position c ^ ((r >> 1) & 3), which makes the kernel's 16-byte
    # shared-memory loads (8 consecutive rows per phase) bank-conflict free.
    word = word.view(rt, kb, 128, 4, 4)
    rows = torch.arange(128, device=q.device)
    perm = (torch.arange(4, device=q.device)[None, :] ^ ((rows[:, None] >> 1) & 3))  # [128, 4]
    sw = torch.empty_like(word)
    sw[:, :, rows[:, None], perm] = word[:, :, rows[:, None], torch.arange(4, device=q.device)[None, :]]
    packed_bytes = sw.contiguous().view(torch.uint8).reshape(rt, kb, 128 * 64)
    gpr = 128 // group_size
    s = sc.view(rt, 128, kb, gpr).permute(0, 2, 1, 3).contiguous()
    s_bytes = s.view(torch.uint8).reshape(rt, kb, 128 * gpr * 2)
    return torch.cat([packed_bytes, s_bytes], dim=-1).reshape(-1).contiguous()


def blob_bytes(n: int, k: int, group_size: int) -> int:
    return (n // 128) * (k // 128) * (8192 + 128 * (128 // group_size) * 2)
