"""Host-side index checks for the kernels' inputs (race / bounds debugging).

``CASCADIA_DEBUG_CHECKS=1`` makes the op wrappers copy index tensors to the
host and verify them before each launch: block-table entries and KV slots
inside the cache, token ids inside the vocabulary, expert ids inside the
expert count, sequence lengths inside the block table.  A violation raises
``IndexCheckError`` on the host; the kernel is never launched with it.  (The
kernels themselves carry no traps or device asserts: a bad index is caught
here, before the GPU sees it.)  Off by default: the checks synchronise.
"""
from __future__ import annotations

import os

import torch

ENABLED = os.environ.get("CASCADIA_DEBUG_CHECKS", "0") not in ("", "0")


class IndexCheckError(ValueError):
    pass


def _host(t: torch.Tensor) -> torch.Tensor:
    return t.detach().to("cpu")


def check_range(name: str, t: torch.Tensor, lo: int, hi: int, allow=()):
    """Every element in [lo, hi) (or one of ``allow``)."""
    if t is None or t.numel() == 0:
        return
    v = _host(t).long()
    bad = (v < lo) | (v >= hi)
    for a in allow:
        bad &= v != a
    if bool(bad.any()):
        i = int(bad.nonzero()[0][0]) if bad.dim() == 1 else bad.nonzero()[0].tolist()
        raise IndexCheckError(f"{name}: value {v.flatten()[bad.flatten()][0].item()} at {i} "
                              f"outside [{lo}, {hi})")


def check_paged(block_tables: torch.Tensor, seq_lens: torch.Tensor, num_blocks: int,
                block: int = 16):
    bt, lens = _host(block_tables).long(), _host(seq_lens).long()
    need = (lens + block - 1) // block
    if bool((need > bt.shape[1]).any()):
        raise IndexCheckError("seq_lens exceed the block table width")
    for b in range(bt.shape[0]):
        check_range(f"block_tables[{b}]", bt[b, :int(need[b])], 0, num_blocks)
