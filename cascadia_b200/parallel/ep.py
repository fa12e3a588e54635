"""Expert parallelism (EP) for the sparse-MoE layers.

Each of the W ranks of an EP group holds E / W routed experts (rank r owns
experts [r * E/W, (r+1) * E/W)) and runs attention for its own sequences
(data-parallel attention, replicated dense weights).  A MoE layer exchanges
token rows twice: (token, expert) pairs go to the expert's owner, results
come back and are combined with the router weights.

Two implementations with the same semantics:

* :meth:`ExpertParallel.moe_a2a` -- ``torch.distributed.all_to_all_single``
  (NCCL on GPUs, gloo on CPUs).  The baseline and the CPU test oracle.
* :meth:`ExpertParallel.moe_fused` -- our kernels (csrc/ep.cu) over NVLink
  peer memory: dispatch = P2P row stores into the owner's receive region,
  the down-projection GEMM's epilogue stores each result row straight into
  the source rank's return region, combine = weighted sum of the returned
  rows.  Symmetric buffers come from ``torch.distributed._symmetric_memory``
  (allocation and peer mapping only; no torch collective runs on this path).

The reference runs every expert of a layer on the stage that owns the layer
(crates/cascadia-engine-sparse-moe/src/runner.rs:929-1216 ``dispatch_expert``,
no EP); this module is the B200 design's replacement for it.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from .. import ops

# Tokens per rank up to this use the grouped small-M expert kernel (decode).
SMALL_M_TOKENS = 64


class ExpertParallel:
    def __init__(self, group, rank: int, world: int, device, num_experts: int, hidden: int,
                 top_k: int, max_tokens: int = 64, fused: Optional[bool] = None):
        assert num_experts % world == 0, "experts must divide evenly over the EP group"
        self.group = group
        self.rank, self.world = rank, world
        self.dev = torch.device(device)
        self.E = num_experts
        self.e_local = num_experts // world
        self.lo = rank * self.e_local
        self.hi = self.lo + self.e_local
        self.hidden = hidden
        self.k = top_k
        self.max_tokens = max_tokens
        self.cap = max_tokens * top_k  # rows one source can send one destination
        # Upper bound on any rank's tokens per call: sizes the grouped GEMM
        # grid (world * row_bound rows per expert at most).  Callers that run
        # smaller batches in lockstep (decode) may lower it.
        self.row_bound = max_tokens
        if fused is None:
            fused = self.dev.type == "cuda" and world > 1
        self.fused = fused
        if fused:
            self._init_symmetric()

    # ------------------------------------------------------------ set-up
    def _init_symmetric(self):
        import torch.distributed._symmetric_memory as symm_mem

        W, cap, H = self.world, self.cap, self.hidden
        gname = self.group.group_name if self.group is not None else dist.group.WORLD.group_name

        def sym(shape, dtype):
            t = symm_mem.empty(shape, dtype=dtype, device=self.dev)
            t.zero_()
            hdl = symm_mem.rendezvous(t, gname)
            ptrs = torch.tensor([int(p) for p in hdl.buffer_ptrs], dtype=torch.int64)
            return t, hdl, ptrs

        self.xbuf, h1, self.xbuf_ptrs = sym((W * cap * H,), torch.bfloat16)
        self.rbuf, h2, self.rbuf_ptrs = sym((W * cap * H,), torch.bfloat16)
        self.meta, h3, self.meta_ptrs = sym((W * cap,), torch.int32)
        self.sig, h4, self.sig_ptrs = sym((64,), torch.int32)
        self._handles = (h1, h2, h3, h4)
        self.epoch = torch.zeros(1, dtype=torch.int32, device=self.dev)
        self.done = torch.zeros(1, dtype=torch.int32, device=self.dev)
        n = self.max_tokens * self.k
        self.dest = torch.zeros(max(1, n), dtype=torch.int32, device=self.dev)
        self.pos = torch.zeros(max(1, n), dtype=torch.int32, device=self.dev)
        self.send_cnt = torch.zeros(W, dtype=torch.int32, device=self.dev)
        self.xp = torch.zeros(W * cap, H, dtype=torch.bfloat16, device=self.dev)
        self.offsets = torch.zeros(self.e_local + 1, dtype=torch.int32, device=self.dev)
        self.src_row = torch.zeros(W * cap, dtype=torch.int32, device=self.dev)
        self.out_rows = torch.zeros(W * cap, dtype=torch.int64, device=self.dev)
        self.total = torch.zeros(1, dtype=torch.int32, device=self.dev)
        torch.cuda.synchronize(self.dev)
        dist.barrier(group=self.group)  # every pad is zero before anyone signals

    def _common(self):
        return (self.xbuf_ptrs, self.rbuf_ptrs, self.meta_ptrs, self.sig_ptrs, self.epoch,
                self.done, ops.status_buffer(self.dev), self.rank, self.world, self.cap,
                self.e_local)

    # ------------------------------------------------------------ forward
    def moe(self, bank, h: torch.Tensor, ids: torch.Tensor, w: torch.Tensor,
            add: Optional[torch.Tensor], out: torch.Tensor) -> torch.Tensor:
        if self.fused:
            return self.moe_fused(bank, h, ids, w, add, out)
        return self.moe_a2a(bank, h, ids, w, add, out)

    def moe_fused(self, bank, h, ids, w, add, out):
        """Dispatch / expert GEMMs / combine over peer memory (all ranks call
        this for every MoE layer, in the same order)."""
        T = h.shape[0]
        assert T <= self.max_tokens, f"{T} tokens > EP capacity {self.max_tokens}"
        assert T <= self.row_bound, f"{T} tokens > the row bound {self.row_bound} set for this call"
        e = ops.ext()
        c = self._common()
        e.ep_dispatch(h, ids, self.dest, self.pos, self.send_cnt, *c)
        e.ep_receive(self.xp, self.offsets, self.src_row, self.out_rows, self.total, *c)
        max_rows = self.world * self.row_bound  # each token reaches an expert at most once
        if self.row_bound <= SMALL_M_TOKENS and bank.gs == 128:
            # Decode: grouped small-M kernel on fp16-prepared rows; the down
            # projection's epilogue still stores into the sources' regions.
            rows = min(self.world * self.row_bound * self.k, self.xp.shape[0])
            x16, xs = ops.moe_prep_fp16(self.xp, rows, rows_dev=self.total)
            act = ops.w4a16_gemv_grouped(x16, xs, bank.gu_blob, 2 * bank.inter, ops.EPI_SILU,
                                         self.offsets, self.e_local, sched=bank.sched[0])
            a16, a_s = ops.moe_prep_fp16(act, rows, rows_dev=self.total)
            ops.w4a16_gemv_grouped(a16, a_s, bank.dn_blob, bank.hidden, ops.EPI_STORE,
                                   self.offsets, self.e_local, out=act[:1, :0],
                                   out_rows=self.out_rows, sched=bank.sched[1])
        else:
            act = ops.w4a16_gemm_grouped(self.xp, bank.gu_blob, 2 * bank.inter, bank.gs,
                                         ops.EPI_SILU, self.offsets, self.e_local, max_rows)
            ops.w4a16_gemm_grouped(act, bank.dn_blob, bank.hidden, bank.gs, ops.EPI_STORE,
                                   self.offsets, self.e_local, max_rows, out_rows=self.out_rows)
        e.ep_combine(w, self.dest, self.pos, add, out, *c)
        ops.LAUNCHES.add(6)
        return out

    def moe_a2a(self, bank, h, ids, w, add, out):
        """Baseline: all-to-all of the routed rows through torch.distributed."""
        T, k = ids.shape
        H = h.shape[1]
        flat = ids.reshape(-1).long()
        dest = flat // self.e_local
        order = torch.argsort(dest, stable=True)
        send_counts = torch.bincount(dest, minlength=self.world)
        send_x = h.index_select(0, (order // k).to(h.device)) if T else h[:0]
        send_e = flat[order].to(torch.int32)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        sc, rc = send_counts.tolist(), recv_counts.tolist()
        recv_x = torch.empty(sum(rc), H, dtype=h.dtype, device=h.device)
        dist.all_to_all_single(recv_x, send_x.contiguous(), rc, sc, group=self.group)
        recv_e = torch.empty(sum(rc), dtype=torch.int32, device=send_e.device)
        dist.all_to_all_single(recv_e, send_e.contiguous(), rc, sc, group=self.group)
        y = expert_ffn(bank, recv_x, (recv_e.long() - self.lo).to(recv_x.device))
        back = torch.empty(sum(sc), H, dtype=y.dtype, device=y.device)
        dist.all_to_all_single(back, y.contiguous(), sc, rc, group=self.group)
        ret = torch.empty(T * k, H, dtype=torch.float32, device=h.device)
        ret[order.to(h.device)] = back.float()
        acc = (ret.view(T, k, H) * w.float().view(T, k, 1).to(h.device)).sum(1)
        if add is not None:
            acc = acc + add.float()
        out.copy_(acc.to(out.dtype))
        return out


def expert_ffn(bank, x: torch.Tensor, le: torch.Tensor) -> torch.Tensor:
    """SwiGLU expert FFN of each row with its local expert id (bf16 out)."""
    n = x.shape[0]
    if n == 0:
        return x.new_zeros(0, bank.hidden)
    if x.device.type == "cuda":
        offsets, perm, inv, xp = ops.moe_permute(le.to(torch.int32).view(n, 1), bank.E, x)
        act = ops.w4a16_gemm_grouped(xp, bank.gu_blob, 2 * bank.inter, bank.gs, ops.EPI_SILU,
                                     offsets, bank.E, n)
        y = ops.w4a16_gemm_grouped(act, bank.dn_blob, bank.hidden, bank.gs, ops.EPI_STORE,
                                   offsets, bank.E, n)
        return y.index_select(0, inv[:n].long())
    from ..ops import reference as ref

    out = torch.empty(n, bank.hidden, dtype=torch.bfloat16)
    for i in range(n):
        e = int(le[i])
        gu = x[i:i + 1].float() @ bank.gu_ref[e].t()
        a = ref.silu_mul(gu[:, :bank.inter], gu[:, bank.inter:]).to(torch.bfloat16)
        out[i] = (a.float() @ bank.dn_ref[e].t()).to(torch.bfloat16)[0]
    return out
