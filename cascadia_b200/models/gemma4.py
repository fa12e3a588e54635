"""Gemma-4 text decoder (HF ``gemma4`` text model).

The reference runs Gemma-4 as a multi-stage OpenVINO chain with cross-KV
frames for the shared-KV layers (crates/cascadia-engine-openvino/src/
gemma4.rs:1-27, engine :1012, builder :1208; docs/architectures/
gemma4-support.md).  Here a model object runs one stage (or all layers) on
our kernels; across pipeline stages each stage hands the next its hidden
rows widened by the per-layer inputs of the later layers and by the K/V rows
of every shared-cache source layer that a later stage reads, which the
receiving stage keeps in mirror pools (``pack_payload`` /
``unpack_payload``):

* layer types: sliding-window attention (head_dim 256, window masked inside
  the attention kernels) and full attention (head_dim 512: the decode
  kernel splits each head's output over two CTAs; prefill of those layers
  runs the decode kernel with one virtual sequence per token);
* q/k RMSNorm (scaled), v RMSNorm (unscaled), attention scale 1;
  ``attention_k_eq_v`` full layers take V from the raw K projection (its
  rows are duplicated in the fused projection);
* sandwich norms around attention and MLP, GeLU-tanh MLP (INT4 GEMM, then
  the activation), per-layer input embeddings (PLE) gated into the residual
  stream after every layer, a per-layer scalar;
* the last ``num_kv_shared_layers`` layers reuse the K/V cache of the last
  earlier layer of their type (no K/V projection, no cache write);
* proportional RoPE on full layers (rotation on the first quarter of the
  frequency pairs, identity on the rest), logits soft-capped.

The mixture-of-experts variant (``enable_moe_block``) adds, beside each
layer's MLP, routed experts fed from the pre-MLP residual: the router
RMS-normalises it (no weight), scales by a learned vector and H^-1/2
(folded into the router rows), softmax top-k, renormalised, times a
per-expert scale; the experts (GeLU-tanh) read their own pre-norm of the
residual, and the two branches are normed separately and summed before the
MLP's post-norm (transformers ``Gemma4TextDecoderLayer``).  On the GPU the
router is the fused top-k gate kernel and the experts run the grouped
small-M / grouped tcgen05 kernels with a store epilogue (GeLU in between).
Caches: one paged pool per head size (256 / 512) over the same block
tables.  The CPU path is the fp32 oracle.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, List, Optional

import torch
import torch.nn.functional as F

from .. import ops
from ..ops import reference as ref
from ..quant import Int4Weight
from ..runtime.kv_cache import BLOCK_SIZE, KVCache
from .config import ModelConfig
from .llama import Batch, LlamaModel, QLinear, _layer_generator, random_int4

SLIDING = "sliding_attention"
FULL = "full_attention"


def gemma_rope_table(theta: float, head_dim: int, rotated_pairs: int, max_pos: int,
                     device) -> torch.Tensor:
    """[max_pos, head_dim] fp32, cos then sin of head_dim / 2 frequencies;
    pairs past ``rotated_pairs`` have frequency 0 (proportional RoPE)."""
    i = torch.arange(rotated_pairs, dtype=torch.float64)
    inv = 1.0 / (theta ** (2 * i / head_dim))
    inv = torch.cat([inv, torch.zeros(head_dim // 2 - rotated_pairs, dtype=torch.float64)])
    ang = torch.outer(torch.arange(max_pos, dtype=torch.float64), inv).float()
    return torch.cat([ang.cos(), ang.sin()], dim=1).to(device)


class DualKVCache(KVCache):
    """Paged K/V for the sliding layers (head_dim d) and, on the same block
    tables, a second pool for the full layers (head_dim d2)."""

    def __init__(self, n1, n2, num_blocks, hkv1, d1, hkv2, d2, device):
        super().__init__(max(1, n1), num_blocks, hkv1, d1, device)
        shape = (max(1, n2), num_blocks, hkv2, BLOCK_SIZE, d2)
        self.k2 = torch.zeros(shape, dtype=torch.bfloat16, device=device)
        self.v2 = torch.zeros(shape, dtype=torch.bfloat16, device=device)

    def gather2(self, layer: int, seq_id: str):
        s = self.seqs[seq_id]
        ids = torch.tensor(s.blocks, dtype=torch.long, device=self.k2.device).clamp_min(0)
        hk = self.k2.shape[2]
        k = self.k2[layer, ids].permute(0, 2, 1, 3).reshape(-1, hk, self.k2.shape[-1])
        v = self.v2[layer, ids].permute(0, 2, 1, 3).reshape(-1, hk, self.v2.shape[-1])
        return k, v


@dataclass
class G4Layer:
    full: bool
    shared: bool            # reuses the cache of layer `cache_idx` (no K/V of its own)
    cache_idx: int          # index in the pool of its head size
    hq: int
    hkv: int
    d: int
    k_eq_v: bool
    in_norm: torch.Tensor
    post_attn_norm: torch.Tensor
    pre_ff_norm: torch.Tensor
    post_ff_norm: torch.Tensor
    qkv: QLinear            # rows q | k | v (v = k rows again when k_eq_v; q only when shared)
    o: QLinear
    q_norm: torch.Tensor
    k_norm: torch.Tensor
    gate_up: QLinear        # rows gate | up
    down: QLinear
    ple_gate: Optional[QLinear]
    ple_proj: Optional[QLinear]
    ple_norm: Optional[torch.Tensor]
    scalar: float
    moe: Optional["G4MoE"] = None


@dataclass
class G4MoE:
    router: torch.Tensor          # [E, H] bf16, scale * H^-1/2 folded into the columns
    expert_scale: torch.Tensor    # [E] fp32
    experts: object               # moe.ExpertBank (gate | up rows, not interleaved)
    post_ff_norm_1: torch.Tensor  # after the MLP branch
    pre_ff_norm_2: torch.Tensor   # expert input
    post_ff_norm_2: torch.Tensor  # after the expert branch


class Gemma4Model(LlamaModel):
    def __init__(self, cfg: ModelConfig, device, tp=None, layer_start: int = 0,
                 layer_end: Optional[int] = None, has_embed: bool = True, has_head: bool = True,
                 **_):
        super().__init__(cfg, device, tp, layer_start, layer_end, has_embed, has_head)
        assert self.tp.size == 1, "Gemma-4: TP=1"
        self.types = list(cfg.layer_types)
        L = cfg.num_layers
        first_shared = L - cfg.num_kv_shared_layers
        self.first_shared = first_shared
        self.spec: List[dict] = []
        self.src_of: Dict[int, int] = {}  # shared layer -> the layer whose cache it reads
        for li in range(L):
            full = self.types[li] == FULL
            shared = cfg.num_kv_shared_layers > 0 and li >= first_shared
            if shared:
                self.src_of[li] = max(j for j in range(first_shared)
                                      if self.types[j] == self.types[li])
            self.spec.append(dict(full=full, shared=shared))
        # Pipeline stages: this stage's pools are its own cache layers plus
        # mirrors of source layers that live on earlier stages (their K/V
        # rows arrive with the hidden rows, see pack_payload).  A stage also
        # forwards the rows of sources that later stages need.
        S, E = self.layer_start, self.layer_end
        owners = [li for li in range(S, E) if not self.spec[li]["shared"]]
        self.mirror_in = sorted({src for li, src in self.src_of.items() if li >= S and src < S})
        self.mirror_out = sorted({src for li, src in self.src_of.items() if li >= E and src < E})
        self.pool: Dict[int, int] = {}
        cnt = {False: 0, True: 0}
        for li in sorted(owners + self.mirror_in):
            full = self.spec[li]["full"]
            self.pool[li] = cnt[full]
            cnt[full] += 1
        for li in range(S, E):
            self.spec[li]["cache_idx"] = self.pool[self.src_of.get(li, li)]
        self.n1, self.n2 = cnt[False], cnt[True]
        self._ple_start = 0
        self.P = cfg.hidden_size_per_layer_input
        self.embed_scale = math.sqrt(cfg.hidden_size)
        self._ple = None
        maxp = min(cfg.max_position, 1 << 16)
        self.cs_local = gemma_rope_table(cfg.rope_theta_local, cfg.head_dim, cfg.head_dim // 2,
                                         maxp, self.device)
        gd = cfg.global_head_dim
        self.cs_global = gemma_rope_table(cfg.rope_theta, gd, int(cfg.global_partial_rotary * gd) // 2,
                                          maxp, self.device)
        self.cos_sin = self.cs_local

    # ------------------------------------------------------------ weights
    def init_random(self, seed: int = 0, std: float = 0.02, gen_device=None):
        cfg = self.cfg
        dev = torch.device(gen_device) if gen_device is not None else self.device
        gs, H, L, P = cfg.group_size, cfg.hidden_size, cfg.num_layers, self.P
        sd = {}
        g = _layer_generator(seed, 100000, dev)
        sd["embed_tokens.weight"] = torch.randn(cfg.vocab_size, H, generator=g, device=dev) * std
        if P:
            sd["embed_tokens_per_layer.weight"] = torch.randn(cfg.vocab_size_per_layer_input, L * P,
                                                              generator=g, device=dev) * std
            sd["per_layer_model_projection.weight"] = torch.randn(L * P, H, generator=g,
                                                                  device=dev) * std
            sd["per_layer_projection_norm.weight"] = torch.ones(P, device=dev)
        sd["norm.weight"] = torch.ones(H, device=dev)
        for li in range(self.layer_start, self.layer_end):
            g = _layer_generator(seed, li, dev)
            p = f"layers.{li}."
            sp = self.spec[li]
            d = cfg.global_head_dim if sp["full"] else cfg.head_dim
            hkv = cfg.num_global_kv_heads if (sp["full"] and cfg.attention_k_eq_v) else cfg.num_kv_heads
            I = cfg.intermediate_size * (2 if (cfg.use_double_wide_mlp and sp["shared"]) else 1)
            r = lambda n, k: torch.randn(n, k, generator=g, device=dev) * std  # noqa: E731
            sd[p + "self_attn.q_proj.weight"] = r(cfg.num_heads * d, H)
            sd[p + "self_attn.k_proj.weight"] = r(hkv * d, H)
            if not (sp["full"] and cfg.attention_k_eq_v):
                sd[p + "self_attn.v_proj.weight"] = r(hkv * d, H)
            sd[p + "self_attn.o_proj.weight"] = r(H, cfg.num_heads * d)
            sd[p + "self_attn.q_norm.weight"] = torch.ones(d, device=dev)
            sd[p + "self_attn.k_norm.weight"] = torch.ones(d, device=dev)
            sd[p + "mlp.gate_proj.weight"] = r(I, H)
            sd[p + "mlp.up_proj.weight"] = r(I, H)
            sd[p + "mlp.down_proj.weight"] = r(H, I)
            for n in ("input_layernorm", "post_attention_layernorm", "pre_feedforward_layernorm",
                      "post_feedforward_layernorm"):
                sd[p + n + ".weight"] = torch.ones(H, device=dev)
            if cfg.gemma_moe:
                E, Im = cfg.num_experts, cfg.moe_intermediate_size
                sd[p + "router.proj.weight"] = r(E, H)
                sd[p + "router.scale"] = torch.ones(H, device=dev)
                sd[p + "router.per_expert_scale"] = torch.ones(E, device=dev)
                sd[p + "experts.gate_up_proj"] = torch.randn(E, 2 * Im, H, generator=g,
                                                             device=dev) * std
                sd[p + "experts.down_proj"] = torch.randn(E, H, Im, generator=g, device=dev) * std
                for n in ("post_feedforward_layernorm_1", "pre_feedforward_layernorm_2",
                          "post_feedforward_layernorm_2"):
                    sd[p + n + ".weight"] = torch.ones(H, device=dev)
            if P:
                sd[p + "per_layer_input_gate.weight"] = r(P, H)
                sd[p + "per_layer_projection.weight"] = r(H, P)
                sd[p + "post_per_layer_input_norm.weight"] = torch.ones(H, device=dev)
            sd[p + "layer_scalar"] = torch.ones(1, device=dev)
        return load_hf_weights(self, sd, prefix="")

    # ------------------------------------------------------------ caches
    def allocate_kv(self, num_blocks: int) -> KVCache:
        cfg = self.cfg
        hkv2 = cfg.num_global_kv_heads if cfg.attention_k_eq_v else cfg.num_kv_heads
        self.kv = DualKVCache(self.n1, self.n2, num_blocks, cfg.num_kv_heads, cfg.head_dim, hkv2,
                              cfg.global_head_dim, self.device)
        return self.kv

    def kv_bytes_per_block(self) -> int:
        cfg = self.cfg
        hkv2 = cfg.num_global_kv_heads if cfg.attention_k_eq_v else cfg.num_kv_heads
        return (KVCache.bytes_per_block(max(1, self.n1), cfg.num_kv_heads, cfg.head_dim) +
                KVCache.bytes_per_block(max(1, self.n2), hkv2, cfg.global_head_dim))

    # ------------------------------------------------------------ forward
    def embed_tokens(self, ids: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Scaled token embeddings; also prepares the per-layer inputs of
        this step (they need the token ids)."""
        cfg = self.cfg
        T = ids.shape[0]
        x = (self.embed.index_select(0, ids.long()).float() *
             torch.tensor(self.embed_scale, dtype=torch.bfloat16).float()).to(torch.bfloat16)
        if out is None:
            out = x
        else:
            out.copy_(x)
        if self.P:
            L, P = cfg.num_layers, self.P
            ple = (self.ple_embed.index_select(0, ids.long()).float() *
                   float(torch.tensor(math.sqrt(P), dtype=torch.bfloat16))).view(T, L, P)
            proj = self.ple_model_proj(out).float() * (cfg.hidden_size ** -0.5)
            proj = proj.to(torch.bfloat16).float().view(T, L, P)
            proj = proj * torch.rsqrt(proj.pow(2).mean(-1, keepdim=True) + cfg.rms_eps) * \
                self.ple_proj_norm.float()
            self._ple = ((proj.to(torch.bfloat16).float() + ple.to(torch.bfloat16).float()) *
                         (2 ** -0.5)).to(torch.bfloat16)
            self._ple_start = 0
        return out

    # ------------------------------------------------ pipeline stage payload
    def _kv_shape(self, li: int):
        cfg = self.cfg
        if self.spec[li]["full"]:
            hkv = cfg.num_global_kv_heads if cfg.attention_k_eq_v else cfg.num_kv_heads
            return hkv, cfg.global_head_dim
        return cfg.num_kv_heads, cfg.head_dim

    def _mirror_width(self, layers) -> int:
        return sum(2 * h * d for h, d in (self._kv_shape(li) for li in layers))

    @property
    def payload_in_width(self) -> int:
        L, P = self.cfg.num_layers, self.P
        return self.cfg.hidden_size + (L - self.layer_start) * P + self._mirror_width(
            self.mirror_in)

    @property
    def payload_out_width(self) -> int:
        L, P = self.cfg.num_layers, self.P
        return self.cfg.hidden_size + (L - self.layer_end) * P + self._mirror_width(
            self.mirror_out)

    def _pool_of(self, li: int):
        kv = self.kv
        kc, vc = (kv.k2, kv.v2) if self.spec[li]["full"] else (kv.k, kv.v)
        return kc, vc, self.pool[li]

    @staticmethod
    def _slot_index(slots: torch.Tensor):
        sl = slots.long()
        return sl // BLOCK_SIZE, sl % BLOCK_SIZE

    def pack_payload(self, hidden: torch.Tensor, batch: Batch) -> torch.Tensor:
        """hidden | per-layer inputs of the later layers | K and V rows (as
        cached: normed, roped) of every source layer that a later stage's
        shared layers read."""
        T = hidden.shape[0]
        L, E = self.cfg.num_layers, self.layer_end
        parts = [hidden]
        if self.P and E < L:
            parts.append(self._ple[:, E - self._ple_start:].reshape(T, -1).to(torch.bfloat16))
        if self.mirror_out:
            blk, off = self._slot_index(batch.slots)
            for src in self.mirror_out:
                kc, vc, p = self._pool_of(src)
                parts.append(kc[p, blk, :, off, :].reshape(T, -1))
                parts.append(vc[p, blk, :, off, :].reshape(T, -1))
        return torch.cat(parts, 1) if len(parts) > 1 else hidden

    def unpack_payload(self, buf: torch.Tensor, batch: Batch,
                       out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Inverse of the previous stage's pack_payload: returns the hidden
        rows, keeps the per-layer inputs (a view of `buf`) and writes the
        mirrored K/V rows into this stage's pools at the batch's slots."""
        cfg = self.cfg
        H, L, S, P = cfg.hidden_size, cfg.num_layers, self.layer_start, self.P
        T = buf.shape[0]
        if out is None:
            out = buf[:, :H].clone()
        else:
            out.copy_(buf[:, :H])
        off = H
        if P:
            n = (L - S) * P
            self._ple = buf[:, off:off + n].reshape(T, L - S, P)
            self._ple_start = S
            off += n
        if self.mirror_in:
            blk, so = self._slot_index(batch.slots)
            for src in self.mirror_in:
                h, d = self._kv_shape(src)
                kc, vc, p = self._pool_of(src)
                kc[p, blk, :, so, :] = buf[:, off:off + h * d].reshape(T, h, d).to(kc.dtype)
                off += h * d
                vc[p, blk, :, so, :] = buf[:, off:off + h * d].reshape(T, h, d).to(vc.dtype)
                off += h * d
        return out

    def _rms(self, x, w, eps=None):
        """RMSNorm in fp32 with the bf16 rounding of the HF model; w None:
        no scale."""
        eps = self.cfg.rms_eps if eps is None else eps
        xf = x.float()
        y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
        if w is not None:
            y = y * w.float()
        return y.to(torch.bfloat16)

    def _norm_to(self, x, w, out):
        if self.device.type == "cuda":
            return ops.rmsnorm(x, w, out, self.cfg.rms_eps)
        out.copy_(self._rms(x, w))
        return out

    def forward(self, batch: Batch, hidden: torch.Tensor) -> torch.Tensor:
        T = hidden.shape[0]
        h = torch.empty_like(hidden)
        t2 = torch.empty_like(hidden)
        for i, lw in enumerate(self.layers):
            self._norm_to(hidden, lw.in_norm, h)
            attn = self._attention_g4(i, lw, h, batch)
            a = lw.o(attn)
            self._norm_to(a, lw.post_attn_norm, t2)
            hidden.copy_((hidden.float() + t2.float()).to(torch.bfloat16))
            self._norm_to(hidden, lw.pre_ff_norm, h)
            gu = lw.gate_up(h)
            I = gu.shape[1] // 2
            act = (F.gelu(gu[:, :I].float(), approximate="tanh") * gu[:, I:].float()).to(
                torch.bfloat16)
            m = lw.down(act)
            if lw.moe is not None:
                m = self._moe_branch(lw.moe, m, hidden)
            self._norm_to(m, lw.post_ff_norm, t2)
            hidden.copy_((hidden.float() + t2.float()).to(torch.bfloat16))
            if lw.ple_gate is not None:
                gte = lw.ple_gate(hidden)
                ple_i = self._ple[:, self.layer_start + i - self._ple_start]
                gte = (F.gelu(gte.float(), approximate="tanh") * ple_i.float()).to(
                    torch.bfloat16)
                pr = lw.ple_proj(gte)
                self._norm_to(pr, lw.ple_norm, t2)
                hidden.copy_((hidden.float() + t2.float()).to(torch.bfloat16))
            if lw.scalar != 1.0:
                hidden.copy_((hidden.float() * lw.scalar).to(torch.bfloat16))
        return hidden

    def _moe_branch(self, mo: G4MoE, mlp_out: torch.Tensor, resid: torch.Tensor) -> torch.Tensor:
        """norm1(MLP output) + norm2(routed experts of the residual)."""
        cfg = self.cfg
        k = cfg.num_experts_per_tok
        T = resid.shape[0]
        h1 = torch.empty_like(mlp_out)
        self._norm_to(mlp_out, mo.post_ff_norm_1, h1)
        xe = torch.empty_like(resid)
        self._norm_to(resid, mo.pre_ff_norm_2, xe)
        bank = mo.experts
        if self.device.type == "cuda":
            rn = torch.empty_like(resid)
            ops.rmsnorm(resid, self._ones_h, rn, cfg.rms_eps)
            ids, w = ops.moe_topk_gate(rn, mo.router, k, 0, True, 1.0)
            w = w * mo.expert_scale.index_select(0, ids.view(-1).long()).view(T, k)
            n = T * k
            I = bank.inter
            if T <= 8 and bank.gs == 128:
                offsets, perm, inv, _ = ops.moe_permute(ids, bank.E)
                x16, xs = ops.moe_prep_fp16(xe, n, perm, k)
                gu = ops.w4a16_gemv_grouped(x16, xs, bank.gu_blob, 2 * I, ops.EPI_STORE,
                                            offsets, bank.E, sched=bank.sched[0])
                act = (F.gelu(gu[:n, :I].float(), approximate="tanh") *
                       gu[:n, I:].float()).to(torch.bfloat16)
                a16, a_s = ops.moe_prep_fp16(act, n)
                y = ops.w4a16_gemv_grouped(a16, a_s, bank.dn_blob, bank.hidden, ops.EPI_STORE,
                                           offsets, bank.E, sched=bank.sched[1])
            else:
                offsets, perm, inv, xp = ops.moe_permute(ids, bank.E, xe)
                gu = ops.w4a16_gemm_grouped(xp, bank.gu_blob, 2 * I, bank.gs, ops.EPI_STORE,
                                            offsets, bank.E, T)
                act = (F.gelu(gu[:, :I].float(), approximate="tanh") *
                       gu[:, I:].float()).to(torch.bfloat16)
                y = ops.w4a16_gemm_grouped(act, bank.dn_blob, bank.hidden, bank.gs,
                                           ops.EPI_STORE, offsets, bank.E, T)
            h2 = torch.empty_like(resid)
            ops.moe_combine(y, inv, w, out=h2)
        else:
            rn = self._rms(resid, None).float()
            probs = torch.softmax(rn @ mo.router.float().t(), dim=-1)
            wt, ids = torch.topk(probs, k, dim=-1)
            wt = wt / wt.sum(-1, keepdim=True) * mo.expert_scale[ids]
            acc = torch.zeros(T, cfg.hidden_size)
            I = bank.inter
            for t in range(T):
                for j in range(k):
                    e = int(ids[t, j])
                    gu = xe[t:t + 1].float() @ bank.gu_ref[e].t()
                    a = (F.gelu(gu[:, :I], approximate="tanh") * gu[:, I:]).to(torch.bfloat16)
                    y = (a.float() @ bank.dn_ref[e].t()).to(torch.bfloat16)
                    acc[t] += float(wt[t, j]) * y[0].float()
            h2 = acc.to(torch.bfloat16)
        t2 = torch.empty_like(resid)
        self._norm_to(h2, mo.post_ff_norm_2, t2)
        return (h1.float() + t2.float()).to(torch.bfloat16)

    def _attention_g4(self, i: int, lw: G4Layer, h: torch.Tensor, batch: Batch) -> torch.Tensor:
        cfg = self.cfg
        T = h.shape[0]
        hq, hkv, d = lw.hq, lw.hkv, lw.d
        kv = self.kv
        kc, vc = (kv.k2, kv.v2) if lw.full else (kv.k, kv.v)
        cs = self.cs_global if lw.full else self.cs_local
        window = 0 if lw.full else cfg.local_window
        qkv = lw.qkv(h)                                   # [T, (hq [+ 2 hkv]) * d]
        if self.device.type == "cuda":
            q_only = lw.shared
            if q_only:
                # Normalise and rotate q only: the pad K/V heads of this
                # buffer are never written to a cache (slots = -1).
                buf = torch.zeros(T, (hq + 2) * d, dtype=torch.bfloat16, device=h.device)
                buf[:, :hq * d] = qkv
                ops.head_rmsnorm(buf, lw.q_norm, lw.q_norm, hq, 0, d, cfg.rms_eps)
                neg = torch.full_like(batch.slots, -1)
                ops.rope_kv_write(buf, batch.positions, cs, neg, kc, vc, lw.cache_idx, hq, 1, d, d)
                q = buf[:, :hq * d]
            else:
                ops.head_rmsnorm(qkv, lw.q_norm, lw.k_norm, hq, hkv, d, cfg.rms_eps)
                ones = torch.ones(d, dtype=torch.bfloat16, device=h.device)
                ops.head_rmsnorm(qkv[:, (hq + hkv) * d:], ones, ones, hkv, 0, d, cfg.rms_eps)
                ops.rope_kv_write(qkv, batch.positions, cs, batch.slots, kc, vc, lw.cache_idx, hq,
                                  hkv, d, d)
                q = qkv[:, :hq * d]
            out = torch.empty(T, hq * d, dtype=torch.bfloat16, device=h.device)
            if batch.is_decode or lw.full:
                # Full layers (head_dim 512) prefill through the decode kernel,
                # one virtual sequence per token.
                if batch.is_decode:
                    bt, lens = batch.block_tables, batch.seq_lens
                else:
                    bt = batch.block_tables.index_select(0, self._tok2seq(batch))
                    lens = batch.positions + 1
                splits, bps = ops.decode_split_plan(T, kc.shape[2], bt.shape[1])
                g = hq // kc.shape[2]
                n = T * kc.shape[2] * splits * g
                part_o = torch.empty(max(1, n * d), dtype=torch.float32, device=h.device)
                part_ml = torch.empty(max(1, n * 2), dtype=torch.float32, device=h.device)
                ops.attn_decode(q, kc, vc, bt, lens, out, lw.cache_idx, splits, bps, part_o,
                                part_ml, 1.0, window)
            else:
                ops.attn_prefill(q, kc, vc, batch.block_tables, batch.tiles, out, lw.cache_idx,
                                 1.0, window)
            return out
        # CPU oracle.
        x = qkv.float()
        q = self._rms(x[:, :hq * d].view(T, hq, d), lw.q_norm).float()
        pos = batch.positions.long()
        q = ref.apply_rope(q, pos, cs, d)
        if not lw.shared:
            k = self._rms(x[:, hq * d:(hq + hkv) * d].view(T, hkv, d), lw.k_norm).float()
            k = ref.apply_rope(k, pos, cs, d)
            v = self._rms(x[:, (hq + hkv) * d:].view(T, hkv, d), None).float()
            slots = batch.slots.long()
            valid = slots >= 0
            sb, so = slots[valid] // BLOCK_SIZE, slots[valid] % BLOCK_SIZE
            kc[lw.cache_idx, sb, :, so] = k[valid].to(torch.bfloat16)
            vc[lw.cache_idx, sb, :, so] = v[valid].to(torch.bfloat16)
        out = torch.empty(T, hq * d, dtype=torch.float32)
        row = 0
        for sid, ql in zip(batch.seq_ids, batch.q_lens):
            kk, vv = (kv.gather2 if lw.full else kv.gather)(lw.cache_idx, sid)
            ctx = int(batch.ctx_len_of(sid))
            o = ref.attention(q[row:row + ql].to(torch.bfloat16), kk[:ctx], vv[:ctx],
                              pos[row:row + ql], 1.0, window)
            out[row:row + ql] = o.reshape(ql, hq * d)
            row += ql
        return out.to(torch.bfloat16)

    def _tok2seq(self, batch: Batch) -> torch.Tensor:
        key = tuple(batch.q_lens)
        cache = getattr(batch, "_tok2seq", None)
        if cache is None or cache[0] != key:
            import numpy as np

            idx = np.repeat(np.arange(len(batch.q_lens)), batch.q_lens)
            batch._tok2seq = (key, torch.from_numpy(idx).to(self.device))
        return batch._tok2seq[1]

    def head(self, hidden_last: torch.Tensor) -> torch.Tensor:
        h = torch.empty_like(hidden_last)
        self._norm_to(hidden_last, self.final_norm, h)
        logits = self.lm_head(h)
        cap = self.cfg.final_logit_softcapping
        if cap:
            logits = (torch.tanh(logits.float() / cap) * cap).to(logits.dtype)
        return logits


def load_hf_weights(model: Gemma4Model, sd: Dict[str, torch.Tensor],
                    prefix: str = "model.") -> Gemma4Model:
    """Fill ``model`` from a HuggingFace Gemma-4 text state dict (float
    weights; projections quantised to INT4 here)."""
    cfg = model.cfg
    gs, dev = cfg.group_size, model.device

    def W(name):
        return sd[prefix + name].float()

    def q4(w):
        return Int4Weight.quantize(w.float(), gs)

    def bf(w):
        return w.to(torch.bfloat16).to(dev)

    model.embed = bf(W("embed_tokens.weight"))
    if model.P:
        model.ple_embed = bf(W("embed_tokens_per_layer.weight"))
        model.ple_model_proj = QLinear(q4(W("per_layer_model_projection.weight")), dev)
        model.ple_proj_norm = bf(W("per_layer_projection_norm.weight"))
    model.layers = []
    model._ones_h = torch.ones(cfg.hidden_size, dtype=torch.bfloat16, device=dev)
    for li in range(model.layer_start, model.layer_end):
        p = f"layers.{li}."
        sp = model.spec[li]
        moe = None
        if cfg.gemma_moe:
            from .moe import ExpertBank

            gu, dn = W(p + "experts.gate_up_proj"), W(p + "experts.down_proj")
            fold = W(p + "router.scale") * cfg.hidden_size ** -0.5
            moe = G4MoE(router=bf(W(p + "router.proj.weight") * fold[None, :]),
                        expert_scale=W(p + "router.per_expert_scale").to(dev),
                        experts=ExpertBank([q4(gu[e]) for e in range(cfg.num_experts)],
                                           [q4(dn[e]) for e in range(cfg.num_experts)], dev,
                                           interleave=False),
                        post_ff_norm_1=bf(W(p + "post_feedforward_layernorm_1.weight")),
                        pre_ff_norm_2=bf(W(p + "pre_feedforward_layernorm_2.weight")),
                        post_ff_norm_2=bf(W(p + "post_feedforward_layernorm_2.weight")))
        full = sp["full"]
        d = cfg.global_head_dim if full else cfg.head_dim
        k_eq_v = full and cfg.attention_k_eq_v
        hkv = cfg.num_global_kv_heads if k_eq_v else cfg.num_kv_heads
        a = p + "self_attn."
        qw, kw = W(a + "q_proj.weight"), W(a + "k_proj.weight")
        if sp["shared"]:
            rows = qw
        else:
            vw = kw if k_eq_v else W(a + "v_proj.weight")
            rows = torch.cat([qw, kw, vw])
        model.layers.append(G4Layer(
            full=full, shared=sp["shared"], cache_idx=sp["cache_idx"], hq=cfg.num_heads,
            hkv=hkv, d=d, k_eq_v=k_eq_v,
            in_norm=bf(W(p + "input_layernorm.weight")),
            post_attn_norm=bf(W(p + "post_attention_layernorm.weight")),
            pre_ff_norm=bf(W(p + "pre_feedforward_layernorm.weight")),
            post_ff_norm=bf(W(p + "post_feedforward_layernorm.weight")),
            qkv=QLinear(q4(rows), dev), o=QLinear(q4(W(a + "o_proj.weight")), dev),
            q_norm=bf(W(a + "q_norm.weight")), k_norm=bf(W(a + "k_norm.weight")),
            gate_up=QLinear(q4(torch.cat([W(p + "mlp.gate_proj.weight"),
                                          W(p + "mlp.up_proj.weight")])), dev),
            down=QLinear(q4(W(p + "mlp.down_proj.weight")), dev),
            ple_gate=QLinear(q4(W(p + "per_layer_input_gate.weight")), dev) if model.P else None,
            ple_proj=QLinear(q4(W(p + "per_layer_projection.weight")), dev) if model.P else None,
            ple_norm=bf(W(p + "post_per_layer_input_norm.weight")) if model.P else None,
            scalar=float(W(p + "layer_scalar").reshape(-1)[0]), moe=moe))
    model.final_norm = bf(W("norm.weight"))
    head = sd.get("lm_head.weight")
    if head is None or cfg.tie_word_embeddings:
        head = sd[prefix + "embed_tokens.weight"]
    model.lm_head = QLinear(q4(head.float()), dev)
    return model
