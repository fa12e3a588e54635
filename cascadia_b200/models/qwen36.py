"""Hybrid Gated-DeltaNet / gated-attention sparse-MoE decoder (Qwen3.5 and
Qwen3.6-35B-A3B; HF ``model_type`` ``qwen3_5_moe``).

The reference runs this model as a chain of stateful OpenVINO stages
(crates/cascadia-engine-openvino/src/qwen36.rs:1-25, ``Qwen36Builder``
:156, ``impl Engine`` :1261; architecture notes in
docs/architectures/qwen3.6.md).  Here every layer runs our sm_100a kernels:

* Gated DeltaNet layers (3 of every 4): one INT4 projection GEMM produces
  q|k|v, the output gate z and the b/a gating inputs; ``gdn_conv`` applies
  the causal depthwise convolution + SiLU in place; ``gdn_recurrent`` runs
  the delta-rule recurrence with the fp32 state in registers and the gated
  RMSNorm fused; the out projection GEMM adds the residual.
* Full-attention layers (every 4th): q|k|v|gate from one INT4 GEMM, per-head
  RMSNorm of q and k, RoPE on the first 64 of 256 dims, paged-KV attention
  (head_dim 256), output * sigmoid(gate), o projection + residual.
* MoE FFN on every layer: softmax top-8 of 256 experts (renormalised), a
  shared expert scaled by sigmoid(w . x).

RMSNorm weights of this family are stored zero-centred (the norm multiplies
by 1 + w); they are folded to 1 + w once at load.  The linear-attention
state (conv rows and the 128x128 fp32 matrix per value head) lives in
:class:`HybridKVCache`, one slot per live sequence, found by the kernels
through the sequence's first KV block.  The CPU path is the fp32 oracle.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Optional

import torch

from .. import ops
from ..ops import reference as ref
from ..quant import Int4Weight
from ..runtime.kv_cache import BLOCK_SIZE, KVCache
from .config import ModelConfig, rope_table
from .llama import Batch, QLinear, _layer_generator, random_int4
from .moe import ExpertBank, MoELayer, MoEModel

KW = 4  # causal conv width


class HybridKVCache(KVCache):
    """Paged K/V for the full-attention layers plus per-sequence recurrent
    state for the linear-attention layers.

    The recurrent state cannot be shared or rewound, so sequences never share
    prefix blocks here and ``truncate`` below the current length is refused.
    Each sequence owns a state slot; ``block_slot[first block]`` maps the
    sequence's first KV block (present in every batch's block table) to it.
    """

    def __init__(self, n_full: int, n_linear: int, num_blocks: int, kv_heads: int, head_dim: int,
                 max_seqs: int, conv_ch: int, hv: int, dk: int, dv: int, device):
        super().__init__(max(1, n_full), num_blocks, kv_heads, head_dim, device)
        self.max_seqs = max_seqs
        self.conv = torch.zeros(max(1, n_linear), max_seqs, KW - 1, conv_ch, dtype=torch.bfloat16,
                                device=device)
        self.rec = torch.zeros(max(1, n_linear), max_seqs, hv, dk, dv, dtype=torch.float32,
                               device=device)
        self.block_slot = torch.zeros(num_blocks, dtype=torch.int32, device=device)
        self.free_slots = list(range(max_seqs - 1, -1, -1))
        self.slot_of: Dict[str, int] = {}

    @staticmethod
    def state_bytes(n_linear: int, conv_ch: int, hv: int, dk: int, dv: int) -> int:
        return n_linear * ((KW - 1) * conv_ch * 2 + hv * dk * dv * 4)

    def add_sequence(self, seq_id: str, shared_prefix=None):
        if not self.free_slots:
            raise RuntimeError(f"no free recurrent-state slot ({self.max_seqs} sequences live)")
        s = super().add_sequence(seq_id, None)
        slot = self.free_slots.pop()
        self.slot_of[seq_id] = slot
        self.conv[:, slot].zero_()
        self.rec[:, slot].zero_()
        return s

    def reserve(self, seq_id: str, new_length: int):
        first = not self.seqs[seq_id].blocks
        super().reserve(seq_id, new_length)
        blocks = self.seqs[seq_id].blocks
        if first and blocks:
            self.block_slot[blocks[0]] = self.slot_of[seq_id]

    def truncate(self, seq_id: str, new_length: int):
        if new_length < self.seqs[seq_id].length:
            raise NotImplementedError("linear-attention state cannot be rewound")
        super().truncate(seq_id, new_length)

    def free_sequence(self, seq_id: str):
        super().free_sequence(seq_id)
        slot = self.slot_of.pop(seq_id, None)
        if slot is not None:
            self.free_slots.append(slot)


@dataclass
class LinearAttn:
    in_proj: QLinear          # [pad(C + Hv*dv + 2*Hv), H]: q|k|v (C) | z | b | a | pad
    conv_w: torch.Tensor      # [C, 4] bf16
    a_log: torch.Tensor       # [Hv] fp32
    dt_bias: torch.Tensor     # [Hv] fp32
    norm_w: torch.Tensor      # [dv] bf16
    out: QLinear              # [H, Hv*dv]


@dataclass
class HybridLayer(MoELayer):
    lin: Optional[LinearAttn] = None
    shared_gate: Optional[torch.Tensor] = None   # [1, H] bf16


class HybridMoEModel(MoEModel):
    def __init__(self, cfg: ModelConfig, device, tp=None, layer_start: int = 0,
                 layer_end: Optional[int] = None, has_embed: bool = True, has_head: bool = True,
                 ep=None):
        super().__init__(cfg, device, tp, layer_start, layer_end, has_embed, has_head,
                         bf16_attention=False, ep=ep)
        self.hk, self.hv = cfg.linear_num_key_heads, cfg.linear_num_value_heads
        self.dk, self.dv = cfg.linear_key_head_dim, cfg.linear_value_head_dim
        assert (self.dk, self.dv) == (128, 128), "the recurrence kernel is built for 128x128 heads"
        assert cfg.linear_conv_kernel_dim == KW
        self.conv_ch = 2 * self.hk * self.dk + self.hv * self.dv
        zw = self.hv * self.dv
        self.proj_n = -(-(self.conv_ch + zw + 2 * self.hv) // 128) * 128
        # Local layer index -> index into the K/V pool (full layers) or the
        # state pool (linear layers).
        self.kv_index: List[int] = []
        self.lin_index: List[int] = []
        nf = nl = 0
        for li in range(self.layer_start, self.layer_end):
            if cfg.is_linear_layer(li):
                self.lin_index.append(nl)
                self.kv_index.append(-1)
                nl += 1
            else:
                self.kv_index.append(nf)
                self.lin_index.append(-1)
                nf += 1
        self.n_full, self.n_linear = nf, nl
        self._seq_start_cache: Dict[tuple, torch.Tensor] = {}

    # ------------------------------------------------------------ weights
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
            lin = qkv = o = None
            if cfg.is_linear_layer(li):
                lin = self._random_linear(g, dev, std)
            else:
                qkv, o = self._init_attention(g, dev, std)
            I = cfg.moe_intermediate_size
            router = (torch.randn(cfg.num_experts, h, generator=g, device=dev) * std).to(
                torch.bfloat16).to(self.device)
            gus, dns = [], []
            lo, hi = (self.ep.lo, self.ep.hi) if self.ep is not None else (0, cfg.num_experts)
            for ei in range(cfg.num_experts):
                gu = Int4Weight.cat_rows([random_int4(I, h, g, dev, std, gs),
                                          random_int4(I, h, g, dev, std, gs)])
                dn = random_int4(h, I, g, dev, std, gs)
                if lo <= ei < hi:
                    gus.append(gu)
                    dns.append(dn)
            bank = ExpertBank(gus, dns, self.device)
            Is = cfg.shared_expert_intermediate_size or I
            gu = Int4Weight.cat_rows([random_int4(Is, h, g, dev, std, gs),
                                      random_int4(Is, h, g, dev, std, gs)])
            shared = (QLinear(gu, self.device, interleave_gate_up=True),
                      QLinear(random_int4(h, Is, g, dev, std, gs), self.device))
            sgate = (torch.randn(1, h, generator=g, device=dev) * std).to(torch.bfloat16).to(
                self.device) if cfg.shared_expert_gate else None
            self.layers.append(HybridLayer(
                in_norm=ones(h), post_norm=ones(h), qkv=qkv, o=o,
                q_norm=None if lin is not None else ones(d),
                k_norm=None if lin is not None else ones(d),
                dense=None, router=router, router_bias=None, experts=bank, shared=shared,
                lin=lin, shared_gate=sgate))
        if self.has_head:
            self.final_norm = ones(h)
            g = _layer_generator(seed, 100001, dev)
            self.lm_head = QLinear(random_int4(cfg.vocab_size, h, g, dev, std, cfg.group_size),
                                   self.device)
        return self

    def _init_attention(self, g, dev, std):
        """Full attention: rows q (Hq*D) | k | v | gate (Hq*D)."""
        cfg = self.cfg
        h, d, gs = cfg.hidden_size, cfg.head_dim, cfg.group_size
        rows = (2 * cfg.num_heads + 2 * cfg.num_kv_heads) * d
        qkv = QLinear(random_int4(rows, h, g, dev, std, gs), self.device)
        o = QLinear(random_int4(h, cfg.num_heads * d, g, dev, std, gs), self.device)
        return qkv, o

    def _random_linear(self, g, dev, std) -> LinearAttn:
        cfg = self.cfg
        h, gs = cfg.hidden_size, cfg.group_size
        w = torch.randn(self.proj_n, h, generator=g, device=dev) * std
        w[self.conv_ch + self.hv * self.dv + 2 * self.hv:] = 0  # padding rows
        conv = (torch.randn(self.conv_ch, KW, generator=g, device=dev) * 0.3).to(torch.bfloat16)
        a_log = torch.empty(self.hv, device=dev).uniform_(1, 16, generator=g).log()
        out = torch.randn(h, self.hv * self.dv, generator=g, device=dev) * std
        return self.make_linear(Int4Weight.quantize(w, gs), conv, a_log,
                                torch.ones(self.hv, device=dev),
                                torch.ones(self.dv, dtype=torch.bfloat16),
                                Int4Weight.quantize(out, gs))

    def make_linear(self, in_proj: Int4Weight, conv_w, a_log, dt_bias, norm_w,
                    out: Int4Weight) -> LinearAttn:
        return LinearAttn(in_proj=QLinear(in_proj, self.device),
                          conv_w=conv_w.to(torch.bfloat16).contiguous().to(self.device),
                          a_log=a_log.float().to(self.device), dt_bias=dt_bias.float().to(self.device),
                          norm_w=norm_w.to(torch.bfloat16).to(self.device),
                          out=QLinear(out, self.device))

    # ------------------------------------------------------------ caches
    def allocate_kv(self, num_blocks: int, max_seqs: int = 64) -> KVCache:
        self.kv = HybridKVCache(self.n_full, self.n_linear, num_blocks, self.hkv, self.d, max_seqs,
                                self.conv_ch, self.hv, self.dk, self.dv, self.device)
        return self.kv

    def kv_bytes_per_block(self) -> int:
        return KVCache.bytes_per_block(max(1, self.n_full), self.hkv, self.d)

    def state_bytes_per_seq(self) -> int:
        return HybridKVCache.state_bytes(self.n_linear, self.conv_ch, self.hv, self.dk, self.dv)

    def save_state(self, batch: Batch):
        """Copies of the batch's recurrent and conv state (the CUDA-graph
        warm-up runs the step several times; each run advances the state)."""
        kv = self.kv
        slots = kv.block_slot.index_select(0, batch.block_tables[:, 0].long()).long()
        return slots, kv.conv.index_select(1, slots), kv.rec.index_select(1, slots)

    def restore_state(self, saved):
        slots, conv, rec = saved
        self.kv.conv.index_copy_(1, slots, conv)
        self.kv.rec.index_copy_(1, slots, rec)

    def _seq_start(self, batch: Batch) -> torch.Tensor:
        key = tuple(batch.q_lens)
        t = self._seq_start_cache.get(key)
        if t is None:
            cu = [0]
            for q in batch.q_lens:
                cu.append(cu[-1] + q)
            t = torch.tensor(cu, dtype=torch.int32, device=self.device)
            if len(self._seq_start_cache) > 256:
                self._seq_start_cache.clear()
            self._seq_start_cache[key] = t
        return t

    # ------------------------------------------------------------ forward
    def forward(self, batch: Batch, hidden: torch.Tensor) -> torch.Tensor:
        h = torch.empty_like(hidden)
        for i, lw in enumerate(self.layers):
            self._norm(hidden, lw.in_norm, h)
            if lw.lin is not None:
                self._linear_attention(self.lin_index[i], lw.lin, h, hidden, batch)
            else:
                qkv = lw.qkv(h)
                self._qk_norm(qkv, lw)
                n_qkv = (self.hq + 2 * self.hkv) * self.d
                attn = self._attention(self.kv_index[i], qkv if self.device.type == "cuda"
                                       else qkv[:, :n_qkv], batch)
                gate = qkv[:, n_qkv:]
                if self.device.type == "cuda":
                    ops.sigmoid_gate(attn, gate)
                else:
                    attn = (attn.float() * torch.sigmoid(gate.float())).to(torch.bfloat16)
                lw.o(attn, ops.EPI_RESID, residual=hidden, out=hidden)
            self._norm(hidden, lw.post_norm, h)
            self._moe(lw, h, hidden)
        return hidden

    def _shared_expert(self, lw, h):
        """Shared expert output and its gate logits w . x (the sigmoid is
        applied by the combine)."""
        out, _ = super()._shared_expert(lw, h)
        if out is None or lw.shared_gate is None:
            return out, None
        if self.device.type == "cuda":
            g = torch.matmul(h, lw.shared_gate.t()).float().view(-1)
        else:
            g = (h.float() @ lw.shared_gate.float().t()).view(-1)
        return out, g

    def _linear_attention(self, si: int, lin: LinearAttn, h: torch.Tensor, hidden: torch.Tensor,
                          batch: Batch):
        T = h.shape[0]
        C, zw = self.conv_ch, self.hv * self.dv
        kv = self.kv
        proj = lin.in_proj(h)  # [T, proj_n]
        if self.device.type == "cuda":
            seq_start = self._seq_start(batch)
            ops.gdn_conv(proj, C, lin.conv_w, kv.conv[si], seq_start, batch.block_tables,
                         kv.block_slot)
            out = torch.empty(T, zw, dtype=torch.bfloat16, device=self.device)
            ops.gdn_recurrent(proj, proj[:, C:], proj[:, C + zw:], lin.a_log, lin.dt_bias,
                              lin.norm_w, kv.rec[si], seq_start, batch.block_tables,
                              kv.block_slot, out, self.hk, self.hv, self.cfg.rms_eps)
        else:
            out = self._linear_attention_cpu(si, lin, proj, batch)
        lin.out(out, ops.EPI_RESID, residual=hidden, out=hidden)

    def _linear_attention_cpu(self, si, lin, proj, batch) -> torch.Tensor:
        """fp32 oracle of the conv + recurrence + gated norm, token by token."""
        C, zw = self.conv_ch, self.hv * self.dv
        hk, hv, dk, dv = self.hk, self.hv, self.dk, self.dv
        kv = self.kv
        out = torch.empty(proj.shape[0], zw, dtype=torch.bfloat16)
        w = lin.conv_w.float()
        row = 0
        for sid, ql in zip(batch.seq_ids, batch.q_lens):
            slot = kv.slot_of[sid]
            hist = kv.conv[si, slot].float()           # [3, C]
            S = kv.rec[si, slot]                        # [hv, dk, dv] (updated in place)
            for t in range(row, row + ql):
                x = proj[t, :C].float()
                acc = (hist * w[:, :KW - 1].t()).sum(0) + x * w[:, KW - 1]
                acc = acc.to(torch.bfloat16).float()
                y = (acc * torch.sigmoid(acc)).to(torch.bfloat16).float()
                hist = torch.cat([hist[1:], x.view(1, C)], 0)
                q = y[:hk * dk].view(hk, dk)
                k = y[hk * dk:2 * hk * dk].view(hk, dk)
                v = y[2 * hk * dk:].view(hv, dv)
                q = q * torch.rsqrt((q * q).sum(-1, keepdim=True) + 1e-6) / dk ** 0.5
                k = k * torch.rsqrt((k * k).sum(-1, keepdim=True) + 1e-6)
                rep = hv // hk
                q, k = q.repeat_interleave(rep, 0), k.repeat_interleave(rep, 0)
                b = proj[t, C + zw:C + zw + hv].float()
                a = proj[t, C + zw + hv:C + zw + 2 * hv].float()
                g = torch.exp(-torch.exp(lin.a_log.float()) * torch.nn.functional.softplus(
                    a + lin.dt_bias.float()))
                beta = torch.sigmoid(b)
                S.mul_(g.view(hv, 1, 1))
                mem = (S * k.unsqueeze(-1)).sum(1)                     # [hv, dv]
                u = (v - mem) * beta.view(hv, 1)
                S.add_(k.unsqueeze(-1) * u.unsqueeze(1))
                o = (S * q.unsqueeze(-1)).sum(1).to(torch.bfloat16).float()   # [hv, dv]
                nrm = (o * torch.rsqrt((o * o).mean(-1, keepdim=True) + self.cfg.rms_eps)).to(
                    torch.bfloat16).float()
                z = proj[t, C:C + zw].float().view(hv, dv)
                yv = lin.norm_w.float() * nrm * (z * torch.sigmoid(z))
                out[t] = yv.reshape(-1).to(torch.bfloat16)
            kv.conv[si, slot] = hist.to(torch.bfloat16)
            row += ql
        return out


def load_hf_weights(model: HybridMoEModel, sd: Dict[str, torch.Tensor],
                    prefix: str = "model.") -> HybridMoEModel:
    """Fill ``model`` from a HuggingFace ``qwen3_5_moe`` text state dict
    (float weights; every projection is quantised to INT4 here).

    Zero-centred RMSNorm weights become 1 + w; the q projection's per-head
    [q | gate] rows are regrouped into q (all heads) ... gate (all heads)
    behind k and v, so one GEMM row holds q | k | v | gate.
    """
    cfg = model.cfg
    gs = cfg.group_size
    dev = model.device
    H, d, hq, hkv = cfg.hidden_size, cfg.head_dim, cfg.num_heads, cfg.num_kv_heads

    def W(name):
        return sd[prefix + name].float()

    def norm1(name):
        return (1.0 + W(name)).to(torch.bfloat16).to(dev)

    def q4(w):
        return Int4Weight.quantize(w.float(), gs)

    model.cos_sin = rope_table(cfg, min(cfg.max_position, 1 << 16), device=dev)
    if model.has_embed:
        model.embed = W("embed_tokens.weight").to(torch.bfloat16).to(dev)
    model.layers = []
    for li in range(model.layer_start, model.layer_end):
        p = f"layers.{li}."
        lin = qkv = o = qn = kn = None
        if cfg.is_linear_layer(li):
            a = p + "linear_attn."
            ip = torch.zeros(model.proj_n, H)
            C, zw, hv = model.conv_ch, model.hv * model.dv, model.hv
            ip[:C] = W(a + "in_proj_qkv.weight")
            ip[C:C + zw] = W(a + "in_proj_z.weight")
            ip[C + zw:C + zw + hv] = W(a + "in_proj_b.weight")
            ip[C + zw + hv:C + zw + 2 * hv] = W(a + "in_proj_a.weight")
            lin = model.make_linear(q4(ip), W(a + "conv1d.weight").reshape(C, KW),
                                    W(a + "A_log"), W(a + "dt_bias"), W(a + "norm.weight"),
                                    q4(W(a + "out_proj.weight")))
        else:
            a = p + "self_attn."
            qg = W(a + "q_proj.weight").view(hq, 2, d, H)
            rows = torch.cat([qg[:, 0].reshape(hq * d, H), W(a + "k_proj.weight"),
                              W(a + "v_proj.weight"), qg[:, 1].reshape(hq * d, H)])
            qkv = QLinear(q4(rows), dev)
            o = QLinear(q4(W(a + "o_proj.weight")), dev)
            qn, kn = norm1(a + "q_norm.weight"), norm1(a + "k_norm.weight")
        m = p + "mlp."
        gu_all, dn_all = W(m + "experts.gate_up_proj"), W(m + "experts.down_proj")
        lo, hi = (model.ep.lo, model.ep.hi) if model.ep is not None else (0, cfg.num_experts)
        bank = ExpertBank([q4(gu_all[e]) for e in range(lo, hi)],
                          [q4(dn_all[e]) for e in range(lo, hi)], dev)
        se = m + "shared_expert."
        shared = (QLinear(q4(torch.cat([W(se + "gate_proj.weight"), W(se + "up_proj.weight")])), dev,
                          interleave_gate_up=True),
                  QLinear(q4(W(se + "down_proj.weight")), dev))
        sgate = W(m + "shared_expert_gate.weight").to(torch.bfloat16).to(dev)
        model.layers.append(HybridLayer(
            in_norm=norm1(p + "input_layernorm.weight"),
            post_norm=norm1(p + "post_attention_layernorm.weight"), qkv=qkv, o=o, q_norm=qn,
            k_norm=kn, dense=None, router=W(m + "gate.weight").to(torch.bfloat16).to(dev),
            router_bias=None, experts=bank, shared=shared, lin=lin, shared_gate=sgate))
    if model.has_head:
        model.final_norm = norm1("norm.weight")
        head = sd.get("lm_head.weight")
        if head is None:
            head = sd[prefix + "embed_tokens.weight"]
        model.lm_head = QLinear(q4(head.float()), dev)
    return model
