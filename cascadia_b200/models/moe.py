"""Sparse-MoE decoder (Qwen3-MoE shape; Kimi-K2-style sigmoid routing and
shared experts are supported by the same layer).

Per layer: RMSNorm -> attention (bf16 projections through cuBLAS, or INT4,
with optional per-head q/k RMSNorm) -> residual -> RMSNorm -> MoE FFN:

    ids, w = topk_gate(h)                      (fused router + top-k kernel)
    perm   = counting sort of (token, slot) by expert; gather rows
    act    = grouped W4A16 GEMM gate_up (+SiLU epilogue), all experts, 1 launch
    y      = grouped W4A16 GEMM down
    out    = residual + sum_j w[t, j] * y[pos(t, j)]  (+ shared expert)

Routing semantics: softmax + top-k + renormalise (Qwen3, norm_topk_prob), or
sigmoid + bias-for-choice + top-k + renormalise x routed_scaling_factor
(Kimi-K2 / DeepSeek-V3; reference crates/cascadia-int4-gemm/src/shell.rs:261-298).
Expert weights are INT4 (group 128 for Qwen3, 32 for Kimi: the reference's F1
expert format, crates/cascadia-int4-gemm/src/kernel.rs:46-70).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional

import torch

from .. import ops
from ..ops import reference as ref
from ..quant import Int4Weight
from .config import ModelConfig, rope_table
from .llama import Batch, LlamaModel, QLinear, TPGroup, _layer_generator, random_int4


# Token counts up to this use the grouped small-M expert kernel (decode).
SMALL_M_TOKENS = 64


# Token counts up to this run the bf16 projections on our tcgen05 GEMM;
# prefill-sized batches go to cuBLAS, which measured 2.5x faster there
# (1.28-1.37 PFLOP/s against 0.48-0.83 for our one-SM tiles at M = 2048:
# a 128 x 256 tile per SM is bound by shared-memory bandwidth; the 2-SM
# cta_group::2 tile is what closes the gap).
BF16_TCGEN05_MAX_M = 256


class BF16Linear:
    """Plain bf16 projection (the MoE config's attention is bf16).  On CUDA,
    decode-sized token counts run our tcgen05 bf16 GEMM (residual add fused
    into its epilogue); prefill-sized ones run cuBLAS."""

    def __init__(self, w: torch.Tensor, device):
        self.w = w.to(torch.bfloat16).to(device).contiguous()
        self.n, self.k = self.w.shape

    def __call__(self, x, epilogue=ops.EPI_STORE, residual=None, out=None):
        if self.w.device.type == "cuda" and x.shape[0] <= BF16_TCGEN05_MAX_M:
            return ops.bf16_gemm(x, self.w, residual if epilogue == ops.EPI_RESID else None, out)
        if self.w.device.type == "cuda":
            y = torch.matmul(x, self.w.t())
            if epilogue == ops.EPI_RESID:
                y = (y.float() + residual.float()).to(torch.bfloat16)
            if out is not None:
                out.copy_(y)
                return out
            return y
        y = (x.float() @ self.w.float().t())
        if epilogue == ops.EPI_RESID:
            y = y + residual.float()
        y = y.to(torch.bfloat16)
        if out is not None:
            out.copy_(y)
            return out
        return y


class ExpertBank:
    """All routed experts of one layer: blobs back to back (GPU) or dequantised
    fp32 weights (CPU oracle)."""

    def __init__(self, gate_up: List[Int4Weight], down: List[Int4Weight], device,
                 interleave: bool = True):
        from . import llama

        self.int4 = (list(gate_up), list(down)) if llama.KEEP_INT4 else None
        self.E = len(gate_up)
        self.inter = gate_up[0].n // 2
        self.hidden = gate_up[0].k
        self.gs = gate_up[0].group_size
        dev = torch.device(device)
        if dev.type == "cuda":
            # Interleaved gate/up rows feed the fused SiLU epilogue; without
            # it the store epilogue gives [gate | up] columns.
            self.gu_blob = torch.cat([w.to(dev).blob(interleave_gate_up=interleave)
                                      for w in gate_up])
            self.dn_blob = torch.cat([w.to(dev).blob() for w in down])
            self.gu_ref = self.dn_ref = None
            # Unit counters of the grouped small-M kernel (dynamic
            # scheduling), one pair per projection of this layer.
            self.sched = torch.zeros(2, 2, dtype=torch.int32, device=dev)
        else:
            self.gu_blob = self.dn_blob = None
            self.gu_ref = [w.dequant_bf16().float() for w in gate_up]
            self.dn_ref = [w.dequant_bf16().float() for w in down]


@dataclass
class MoELayer:
    in_norm: torch.Tensor
    post_norm: torch.Tensor
    qkv: object
    o: object
    q_norm: Optional[torch.Tensor]
    k_norm: Optional[torch.Tensor]
    dense: Optional[tuple]            # (gate_up QLinear, down QLinear) for dense layers
    router: Optional[torch.Tensor]    # [E, H] bf16
    router_bias: Optional[torch.Tensor]
    experts: Optional[ExpertBank]
    shared: Optional[tuple]           # (gate_up QLinear, down QLinear)


class MoEModel(LlamaModel):
    def __init__(self, cfg: ModelConfig, device, tp: Optional[TPGroup] = None,
                 layer_start: int = 0, layer_end: Optional[int] = None,
                 has_embed: bool = True, has_head: bool = True, bf16_attention: bool = True,
                 ep=None):
        super().__init__(cfg, device, tp, layer_start, layer_end, has_embed, has_head)
        assert self.tp.size == 1, "MoE model: expert parallelism replaces TP (see parallel.ep)"
        self.bf16_attention = bf16_attention
        # parallel.ep.ExpertParallel: this rank holds experts [ep.lo, ep.hi)
        # of every MoE layer and attends over its own sequences.
        self.ep = ep
        self.layers: List[MoELayer] = []

    def init_random(self, seed: int = 0, std: float = 0.02, gen_device=None):
        cfg = self.cfg
        dev = torch.device(gen_device) if gen_device is not None else self.device
        gs = cfg.group_size
        h, d = cfg.hidden_size, cfg.head_dim
        self.cos_sin = rope_table(cfg, min(cfg.max_position, 1 << 16), device=self.device)
        if self.has_embed or (self.has_head and cfg.tie_word_embeddings):
            g = _layer_generator(seed, 100000, dev)
            self.embed = (torch.randn(cfg.vocab_size, h, generator=g, device=dev) * std).to(
                torch.bfloat16).to(self.device)
        ones = lambda n: torch.ones(n, dtype=torch.bfloat16, device=self.device)  # noqa: E731
        for li in range(self.layer_start, self.layer_end):
            g = _layer_generator(seed, li, dev)
            qkv, o = self._init_attention(g, dev, std)
            dense = router = bias = bank = shared = None
            if li < cfg.first_k_dense_replace:
                I = cfg.intermediate_size
                gu = Int4Weight.cat_rows([random_int4(I, h, g, dev, std, gs),
                                          random_int4(I, h, g, dev, std, gs)])
                dense = (QLinear(gu, self.device, interleave_gate_up=True),
                         QLinear(random_int4(h, I, g, dev, std, gs), self.device))
            else:
                I = cfg.moe_intermediate_size
                router = (torch.randn(cfg.num_experts, h, generator=g, device=dev) * std).to(
                    torch.bfloat16).to(self.device)
                if cfg.router == "sigmoid":
                    bias = (torch.randn(cfg.num_experts, generator=g, device=dev) * 0.1).float().to(
                        self.device)
                gus, dns = [], []
                lo, hi = (self.ep.lo, self.ep.hi) if self.ep is not None else (0, cfg.num_experts)
                for ei in range(cfg.num_experts):
                    # Every expert is drawn (the generator stream stays the
                    # same for every EP size); only the local ones are kept.
                    gu = Int4Weight.cat_rows([random_int4(I, h, g, dev, std, gs),
                                              random_int4(I, h, g, dev, std, gs)])
                    dn = random_int4(h, I, g, dev, std, gs)
                    if lo <= ei < hi:
                        gus.append(gu)
                        dns.append(dn)
                bank = ExpertBank(gus, dns, self.device)
                del gus, dns
                if cfg.num_shared_experts:
                    Is = I * cfg.num_shared_experts
                    gu = Int4Weight.cat_rows([random_int4(Is, h, g, dev, std, gs),
                                              random_int4(Is, h, g, dev, std, gs)])
                    shared = (QLinear(gu, self.device, interleave_gate_up=True),
                              QLinear(random_int4(h, Is, g, dev, std, gs), self.device))
            self.layers.append(MoELayer(
                in_norm=ones(h), post_norm=ones(h), qkv=qkv, o=o,
                q_norm=ones(d) if cfg.qk_norm else None, k_norm=ones(d) if cfg.qk_norm else None,
                dense=dense, router=router, router_bias=bias, experts=bank, shared=shared))
        if self.has_head:
            self.final_norm = ones(h)
            g = _layer_generator(seed, 100001, dev)
            self.lm_head = QLinear(random_int4(cfg.vocab_size, h, g, dev, std, gs), self.device)
        return self

    def _init_attention(self, g, dev, std):
        """(qkv, o) projections of one layer, drawn from the layer generator."""
        cfg = self.cfg
        h, d, gs = cfg.hidden_size, cfg.head_dim, cfg.group_size
        qkv_rows = (cfg.num_heads + 2 * cfg.num_kv_heads) * d
        if self.bf16_attention:
            qkv = BF16Linear(torch.randn(qkv_rows, h, generator=g, device=dev) * std, self.device)
            o = BF16Linear(torch.randn(h, cfg.num_heads * d, generator=g, device=dev) * std,
                           self.device)
        else:
            qkv = QLinear(random_int4(qkv_rows, h, g, dev, std, gs), self.device)
            o = QLinear(random_int4(h, cfg.num_heads * d, g, dev, std, gs), self.device)
        return qkv, o

    # ------------------------------------------------------------ forward
    def forward(self, batch: Batch, hidden: torch.Tensor) -> torch.Tensor:
        h = torch.empty_like(hidden)
        for i, lw in enumerate(self.layers):
            self._norm(hidden, lw.in_norm, h)
            qkv = lw.qkv(h)
            if lw.q_norm is not None:
                self._qk_norm(qkv, lw)
            attn = self._attention(i, qkv, batch)
            lw.o(attn, ops.EPI_RESID, residual=hidden, out=hidden)
            self._norm(hidden, lw.post_norm, h)
            if lw.dense is not None:
                act = lw.dense[0](h, ops.EPI_SILU)
                lw.dense[1](act, ops.EPI_RESID, residual=hidden, out=hidden)
            else:
                self._moe(lw, h, hidden)
        return hidden

    def _qk_norm(self, qkv: torch.Tensor, lw: MoELayer):
        """Per-head RMSNorm of q and k (Qwen3) applied in place before RoPE."""
        T = qkv.shape[0]
        hq, hkv, d = self.hq, self.hkv, self.d
        if self.device.type == "cuda":
            ops.head_rmsnorm(qkv, lw.q_norm, lw.k_norm, hq, hkv, d, self.cfg.rms_eps)
            return
        for lo, nh, w in ((0, hq, lw.q_norm), (hq * d, hkv, lw.k_norm)):
            part = qkv[:, lo:lo + nh * d]
            x = part.float().view(T, nh, d)
            part.copy_(ref.rmsnorm(x, w, self.cfg.rms_eps).to(torch.bfloat16).view(T, nh * d))

    def _shared_expert(self, lw: MoELayer, h: torch.Tensor):
        """(output of the layer's shared expert(s) or None, fp32 gate logits
        [T] or None); the combine adds sigmoid(gate) * output."""
        if lw.shared is None:
            return None, None
        return lw.shared[1](lw.shared[0](h, ops.EPI_SILU)), None

    @staticmethod
    def _gated(shared_out, gate):
        if shared_out is None or gate is None:
            return shared_out
        return (shared_out.float() * torch.sigmoid(gate.float()).view(-1, 1)).to(torch.bfloat16)

    # Every this many eager MoE layer calls, the tokens routed to each expert
    # are added to the expert-load histogram (a device-to-host copy of E
    # counts; never inside a CUDA-graph capture).  0 turns it off.
    expert_load_every = 16

    def _record_expert_load(self, ids: torch.Tensor, num_experts: int):
        every = self.expert_load_every
        if every <= 0 or (ids.is_cuda and torch.cuda.is_current_stream_capturing()):
            return
        self._moe_calls = getattr(self, "_moe_calls", 0) + 1
        if (self._moe_calls - 1) % every:
            return
        from .. import metrics

        counts = torch.bincount(ids.reshape(-1).long(), minlength=num_experts).cpu().tolist()
        hist = metrics.EXPERT_LOAD.labels(model=self.cfg.arch)
        for c in counts:
            hist.observe(c)

    def _moe(self, lw: MoELayer, h: torch.Tensor, hidden: torch.Tensor):
        cfg = self.cfg
        k = cfg.num_experts_per_tok
        scoring = 0 if cfg.router == "softmax" else 1
        bank = lw.experts
        shared_out, shared_gate = self._shared_expert(lw, h)
        if self.ep is not None:
            if self.device.type == "cuda":
                ids, w = ops.moe_topk_gate(h, lw.router, k, scoring, cfg.norm_topk_prob,
                                           cfg.routed_scaling_factor, lw.router_bias)
            else:
                ids, w = ref_topk_gate(h, lw.router, lw.router_bias, k, scoring,
                                       cfg.norm_topk_prob, cfg.routed_scaling_factor)
            self._record_expert_load(ids, bank.E if bank is not None else cfg.num_experts)
            so = self._gated(shared_out, shared_gate)
            add = hidden if so is None else (hidden.float() + so.float()).to(torch.bfloat16)
            self.ep.moe(bank, h, ids, w.float(), add, hidden)
            return
        if self.device.type == "cuda":
            ids, w = ops.moe_topk_gate(h, lw.router, k, scoring, cfg.norm_topk_prob,
                                       cfg.routed_scaling_factor, lw.router_bias)
            self._record_expert_load(ids, bank.E)
            T = h.shape[0]
            if T <= SMALL_M_TOKENS and bank.gs == 128:
                # Decode: a few rows per expert -> grouped small-M kernel on
                # fp16-prepared activations (gathered into expert order).
                offsets, perm, inv, _ = ops.moe_permute(ids, bank.E)
                n = T * k
                x16, xs = ops.moe_prep_fp16(h, n, perm, k)
                act = ops.w4a16_gemv_grouped(x16, xs, bank.gu_blob, 2 * bank.inter,
                                             ops.EPI_SILU, offsets, bank.E, sched=bank.sched[0])
                a16, a_s = ops.moe_prep_fp16(act, n)
                y = ops.w4a16_gemv_grouped(a16, a_s, bank.dn_blob, bank.hidden, ops.EPI_STORE,
                                           offsets, bank.E, sched=bank.sched[1])
            else:
                offsets, perm, inv, xp = ops.moe_permute(ids, bank.E, h)
                act = ops.w4a16_gemm_grouped(xp, bank.gu_blob, 2 * bank.inter, bank.gs,
                                             ops.EPI_SILU, offsets, bank.E, T)
                y = ops.w4a16_gemm_grouped(act, bank.dn_blob, bank.hidden, bank.gs,
                                           ops.EPI_STORE, offsets, bank.E, T)
            ops.moe_combine(y, inv, w, add=hidden, out=hidden, shared=shared_out,
                            shared_gate=shared_gate)
            return
        # CPU oracle.
        ids, w = ref_topk_gate(h, lw.router, lw.router_bias, k, scoring, cfg.norm_topk_prob,
                               cfg.routed_scaling_factor)
        self._record_expert_load(ids, bank.E)
        out = torch.zeros(h.shape[0], cfg.hidden_size)
        for t in range(h.shape[0]):
            for j in range(k):
                e = int(ids[t, j])
                gu = h[t:t + 1].float() @ bank.gu_ref[e].t()
                a = ref.silu_mul(gu[:, :bank.inter], gu[:, bank.inter:]).to(torch.bfloat16)
                y = (a.float() @ bank.dn_ref[e].t()).to(torch.bfloat16)
                out[t] += float(w[t, j]) * y[0].float()
        so = self._gated(shared_out, shared_gate)
        if so is not None:
            out += so.float()
        hidden.copy_((hidden.float() + out).to(torch.bfloat16))


def ref_topk_gate(h, wg, bias, k, scoring, norm_topk, routed_scale):
    logits = h.float() @ wg.float().t()
    if scoring == 0:
        scores = torch.softmax(logits, dim=-1)
        sel = scores
    else:
        scores = torch.sigmoid(logits)
        sel = scores + (bias.float() if bias is not None else 0.0)
    ids = torch.topk(sel, k, dim=-1).indices
    w = torch.gather(scores, 1, ids)
    if norm_topk:
        w = w / w.sum(-1, keepdim=True)
    return ids.to(torch.int32), w * routed_scale
