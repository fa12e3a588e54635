"""Tensor-parallel communication for the dense model.

Two paths, same semantics (sum of row-parallel partials over the TP group):

* ``TPGroup`` (models.llama): NCCL all-reduce, the baseline / prefill path;
* ``FusedTP``: our ``ar_rmsnorm`` kernel over NVLink peer memory.  The
  row-parallel GEMM writes its partial straight into a symmetric buffer (the
  same allocation mapped on every GPU of the group); one kernel then signals,
  waits (bounded) for the peers, sums the partials with P2P loads, adds the
  residual and applies the next RMSNorm.  Used for decode-sized token counts.
* ``FusedTP(multimem=True)``: as the default path, but the partials are
  summed by ``multimem.ld_reduce`` on the buffer's NVLink multicast address
  (NVLS: the NVSwitch adds the ranks' rows and returns one sum), so each
  rank reads M x H once instead of once per peer.
* ``FusedTP(push=True)``: the row-parallel GEMM itself stores each finished
  output tile into every rank's receive slot for this rank (plain P2P stores
  from the GEMM epilogue, so the transfer overlaps the rest of the GEMM) and
  its last tile raises this rank's flag in every rank's signal pad; the
  following kernel waits for the flags and reads only local memory.

Symmetric allocation and peer mapping come from
``torch.distributed._symmetric_memory`` (plumbing only: no torch collective
runs on this path).  The signal pad is our own zeroed int32 symmetric tensor.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from .. import ops


class FusedTP:
    def __init__(self, group, rank: int, world: int, device, hidden: int, max_tokens: int = 256,
                 push: bool = False, multimem: bool = False):
        import torch.distributed._symmetric_memory as symm_mem

        self.rank, self.world = rank, world
        self.dev = torch.device(device)
        self.hidden = hidden
        self.max_tokens = max_tokens
        self.buf = symm_mem.empty((2, max_tokens, hidden), dtype=torch.bfloat16, device=self.dev)
        self.buf.zero_()
        gname = group.group_name if group is not None else dist.group.WORLD.group_name
        hdl = symm_mem.rendezvous(self.buf, gname)
        self.sig = symm_mem.empty((8,), dtype=torch.int32, device=self.dev)
        self.sig.zero_()
        shdl = symm_mem.rendezvous(self.sig, gname)
        self.buf_ptrs = torch.tensor([int(p) for p in hdl.buffer_ptrs], dtype=torch.int64)
        self.sig_ptrs = torch.tensor([int(p) for p in shdl.buffer_ptrs], dtype=torch.int64)
        self.mc_ptr = 0
        if multimem:
            if not (hdl.has_multicast_support and int(hdl.multicast_ptr)):
                raise RuntimeError("multimem all-reduce asked for, but this group's symmetric "
                                   "memory has no NVLink multicast object (NVLS)")
            self.mc_ptr = int(hdl.multicast_ptr)
        self.epoch = torch.zeros(1, dtype=torch.int32, device=self.dev)
        self.done = torch.zeros(1, dtype=torch.int32, device=self.dev)
        self._handles = (hdl, shdl)
        self.push = push
        if push:
            # recv[parity, src rank, token, hidden] on every rank.
            self.recv = symm_mem.empty((2, world, max_tokens, hidden), dtype=torch.bfloat16,
                                       device=self.dev)
            self.recv.zero_()
            rhdl = symm_mem.rendezvous(self.recv, gname)
            base = [int(p) for p in rhdl.buffer_ptrs]
            slot = max_tokens * hidden * 2  # bytes of one (parity, src) slot
            # Where this rank's GEMM stores (every rank's slot for this rank)
            # and where this rank reads (its own slots of every source).
            self.push_out = [torch.tensor([base[q] + (b * world + rank) * slot
                                           for q in range(world)], dtype=torch.int64)
                             for b in range(2)]
            self.push_slots = [torch.tensor([base[rank] + (b * world + p) * slot
                                             for p in range(world)], dtype=torch.int64)
                               for b in range(2)]
            self.push_done = torch.zeros(1, dtype=torch.int32, device=self.dev)
            self._handles = (hdl, shdl, rhdl)
        torch.cuda.synchronize(self.dev)
        dist.barrier(group=group)  # every pad is zero before anyone signals

    def gemm_push(self, lin, x: torch.Tensor, slot: int) -> None:
        """Row-parallel GEMM (an INT4 QLinear) whose output goes straight
        into every rank's receive slot `slot` for this rank."""
        e = ops.ext()
        m = x.shape[0]
        ws = ops.default_workspace(x.device)
        mt = 16 if m <= 16 else 32 if m <= 32 else 64 if m <= 64 else 128
        tt = -(-m // mt)
        ws.ensure(8 * tt * mt * lin.n, tt * (lin.n // 128))
        e.w4a16_gemm_push(x, lin.blob, lin.n, lin.group_size, self.push_out[slot], self.hidden,
                          self.sig_ptrs, self.rank, self.push_done, self.epoch, ws.ws,
                          ws.counters, ops.status_buffer(self.dev))
        ops.LAUNCHES.add(1)

    def allreduce_pushed(self, slot: int, m: int, residual: Optional[torch.Tensor],
                         weight: Optional[torch.Tensor], out: torch.Tensor, eps: float):
        """As allreduce(), for partials a pushing GEMM delivered into the
        local slots of `slot`."""
        ops.ext().ar_rmsnorm_pushed(self.push_slots[slot], self.sig_ptrs, self.epoch, self.done,
                                    ops.status_buffer(self.dev), self.rank, self.world, m,
                                    self.hidden, residual, weight, out, eps)
        ops.LAUNCHES.add(1)
        return out

    def partial_out(self, slot: int, m: int) -> torch.Tensor:
        return self.buf[slot, :m]

    def allreduce(self, slot: int, m: int, residual: Optional[torch.Tensor],
                  weight: Optional[torch.Tensor], out: torch.Tensor, eps: float):
        """out = rmsnorm(residual + sum_ranks(partial[slot])) * weight; the
        residual stream is updated in place.  weight=None: out = the sum."""
        ops.ext().ar_rmsnorm(self.buf_ptrs, slot * self.max_tokens * self.hidden * 2,
                             self.sig_ptrs, self.epoch, self.done,
                             ops.status_buffer(self.dev), self.rank, self.world, m, self.hidden,
                             residual, weight, out, eps, self.mc_ptr)
        ops.LAUNCHES.add(1)
        return out
