"""GLM-5 (HF ``glm_moe_dsa``): MLA attention restricted by a DSA lightning
indexer, sigmoid + bias routed MoE with a shared expert, dense first layers.

The reference's GLM-5 shell (crates/cascadia-engine-sparse-moe/src/glm/:
MLA ``attn.rs:163``, indexer ``indexer.rs:50-190``, router ``gate.rs:24``;
architecture notes docs/architectures/glm5.md) runs on CPU.  Here:

* MLA is the absorbed-latent decode kernel of the Kimi-K2 path
  (``csrc/mla.cu``) with GLM-5's head widths (nope 192, v 256).
* The indexer scores every cached position of a query token,
  ``score[p] = sum_h w_h relu(q_h . k_p)`` (``dsa_scores`` kernel over a paged
  cache of 128-wide index keys); the top-``index_topk`` threshold per token
  selects the positions the attention kernel may use (others get -inf).
  With a context of at most ``index_topk`` tokens this is dense attention.
* IndexShare: layers marked "shared" reuse the selection of the previous
  indexer layer (only "full" layers own an indexer).

Checkpoints rotate the rope halves of q and k NeoX-style; the loader
permutes those rows into the interleaved pair order the MLA kernels rotate
(the q.k products are unchanged by a shared permutation).  The indexer's own
rope stays split-half, applied with torch.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, Optional

import torch
import torch.nn.functional as F

from .. import ops
from ..quant import Int4Weight
from ..runtime.kv_cache import BLOCK_SIZE
from .config import rope_table
from .llama import Batch, QLinear, _layer_generator, random_int4
from .mla import LATENT, ROPE, ROW, Int4Pad, LatentKVCache, MLAAttention, MLAModel
from .moe import ExpertBank, MoELayer


@dataclass
class Indexer:
    wq_b: QLinear            # [Hi * 128, q_lora]
    wk: QLinear              # [128, H]
    k_norm_w: torch.Tensor   # [128] fp32 (LayerNorm weight)
    k_norm_b: torch.Tensor   # [128] fp32 (LayerNorm bias)
    w_proj: torch.Tensor     # [Hi, H] bf16


@dataclass
class DSAAttention(MLAAttention):
    indexer: Optional[Indexer] = None


def rope_half(x: torch.Tensor, pos: torch.Tensor, cos_sin: torch.Tensor) -> torch.Tensor:
    """NeoX rotation of the last dim (64): pairs (x[i], x[i + 32])."""
    half = x.shape[-1] // 2
    cs = cos_sin[pos].float()
    shape = [cs.shape[0]] + [1] * (x.dim() - 2) + [half]
    cos, sin = cs[:, :half].reshape(shape), cs[:, half:].reshape(shape)
    x1, x2 = x[..., :half], x[..., half:]
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1)


class GLM5Model(MLAModel):
    def __init__(self, cfg, device, **kw):
        super().__init__(cfg, device, **kw)
        assert cfg.is_dsa and cfg.index_head_dim == 128
        if not cfg.layer_has_indexer(self.layer_start):
            # An IndexShare layer reuses the selection of the indexer layer
            # before it, which a stage that starts with it does not have.
            raise ValueError(f"a GLM-5 stage must start at an indexer layer, not layer "
                             f"{self.layer_start} (indexer_types 'shared')")
        self.hi = cfg.index_n_heads
        # local layer -> slot in the index-key cache (-1: IndexShare layer)
        self.idx_slot = []
        n = 0
        for li in range(self.layer_start, self.layer_end):
            if cfg.layer_has_indexer(li):
                self.idx_slot.append(n)
                n += 1
            else:
                self.idx_slot.append(-1)
        self.n_idx = n
        self._sel = None

    # ------------------------------------------------------------ weights
    def _init_attention(self, g, dev, std):
        attn, o = super()._init_attention(g, dev, std)
        cfg = self.cfg
        h, gs = cfg.hidden_size, cfg.group_size
        li = self.layer_start + len(self.layers)
        ind = None
        if cfg.layer_has_indexer(li):
            ind = Indexer(
                wq_b=QLinear(random_int4(self.hi * 128, cfg.q_lora_rank, g, dev, std, gs), self.device),
                wk=QLinear(random_int4(128, h, g, dev, std, gs), self.device),
                k_norm_w=torch.ones(128, device=self.device),
                k_norm_b=torch.zeros(128, device=self.device),
                w_proj=(torch.randn(self.hi, h, generator=g, device=dev) * std).to(
                    torch.bfloat16).to(self.device))
        return DSAAttention(**{f: getattr(attn, f) for f in attn.__dataclass_fields__},
                            indexer=ind), o

    def allocate_kv(self, num_blocks: int):
        super().allocate_kv(num_blocks)
        # One spare block at the end takes the keys of rows without a slot.
        self.kv.ik = torch.zeros(max(1, self.n_idx), num_blocks + 1, BLOCK_SIZE, 128,
                                 dtype=torch.bfloat16, device=self.device)
        return self.kv

    def kv_bytes_per_block(self) -> int:
        return super().kv_bytes_per_block() + self.n_idx * BLOCK_SIZE * 128 * 2

    # ------------------------------------------------------------ forward
    def forward(self, batch: Batch, hidden: torch.Tensor) -> torch.Tensor:
        self._sel = None
        return super().forward(batch, hidden)

    def _mla(self, li: int, a: DSAAttention, x: torch.Tensor, batch: Batch) -> torch.Tensor:
        q, c, kr, qa_n = self._q_and_kv(a, x)
        if a.indexer is not None:
            self._sel = self._index(self.idx_slot[li], a.indexer, x, qa_n, batch)
        sel = self._sel
        if self.device.type == "cuda":
            return self._mla_gpu(li, a, q, c, kr, batch, sel)
        return self._mla_cpu(li, a, q, c, kr, batch, sel)

    def _index(self, slot: int, ind: Indexer, x: torch.Tensor, qa_n: torch.Tensor, batch: Batch):
        """(scores [T, ld] fp32, thresholds [T]): position p of token t is
        selected iff scores[t, p] >= thresholds[t]."""
        T = x.shape[0]
        hi, k = self.hi, self.cfg.index_topk
        pos = batch.positions.long()
        iq = ind.wq_b(qa_n).float().view(T, hi, 128)
        iq = torch.cat([rope_half(iq[..., :ROPE], pos, self.cos_sin), iq[..., ROPE:]], -1)
        ik = F.layer_norm(ind.wk(x).float(), (128,), ind.k_norm_w, ind.k_norm_b, 1e-6)
        ik = torch.cat([rope_half(ik[:, :ROPE], pos, self.cos_sin), ik[:, ROPE:]], -1)
        slots = batch.slots.long()
        cache = self.kv.ik[slot]
        # Rows without a slot (-1) go to the spare block at the end (no
        # host-side filtering: this also runs inside CUDA graphs).
        spare = (cache.shape[0] - 1) * BLOCK_SIZE
        cache.view(-1, 128).index_copy_(0, torch.where(slots >= 0, slots, spare),
                                        ik.to(torch.bfloat16))
        if self.device.type == "cuda":
            wts = torch.matmul(x, ind.w_proj.t()).float()
        else:
            wts = x.float() @ ind.w_proj.float().t()
        wts = wts * (hi ** -0.5) * (128 ** -0.5)
        if self.device.type == "cuda":
            bt, lens = self._virtual_seqs(batch)
            ld = bt.shape[1] * BLOCK_SIZE
            scores = torch.empty(T, ld, dtype=torch.float32, device=x.device)
            ops.ext().dsa_scores(iq.to(torch.bfloat16).contiguous(), wts.contiguous(), self.kv.ik,
                                 bt, lens, scores, slot)
            ops.LAUNCHES.add(1)
        else:
            ld = max(batch.ctx_lens)
            scores = torch.full((T, ld), float("-inf"))
            r = 0
            for sid, ql in zip(batch.seq_ids, batch.q_lens):
                ctx = int(batch.ctx_len_of(sid))
                s = self.kv.seqs[sid]
                ids = torch.tensor(s.blocks, dtype=torch.long)
                keys = cache[ids].reshape(-1, 128)[:ctx].float()
                qq = iq[r:r + ql]                                           # [ql, hi, 128]
                sc = torch.relu(torch.einsum("qhd,td->qht", qq, keys))
                sc = torch.einsum("qht,qh->qt", sc, wts[r:r + ql])
                causal = torch.arange(ctx)[None, :] > pos[r:r + ql, None]
                scores[r:r + ql, :ctx] = sc.masked_fill(causal, float("-inf"))
                r += ql
        if scores.shape[1] <= k:
            thr = torch.full((T,), float("-inf"), device=scores.device)
        else:
            thr = torch.topk(scores, k, dim=1).values[:, -1].contiguous()
        return scores, thr


def load_hf_weights(model: GLM5Model, sd: Dict[str, torch.Tensor],
                    prefix: str = "model.") -> GLM5Model:
    """Fill ``model`` from a HuggingFace ``glm_moe_dsa`` state dict (float
    weights; projections quantised to INT4 here).  The rope rows of q_b and
    kv_a are permuted from NeoX halves into interleaved pairs."""
    cfg = model.cfg
    gs, dev = cfg.group_size, model.device
    H, hq = cfg.hidden_size, cfg.num_heads
    nope, vd = cfg.qk_nope_head_dim, cfg.v_head_dim
    perm = torch.stack([torch.arange(ROPE // 2), torch.arange(ROPE // 2) + ROPE // 2], 1).reshape(-1)

    def W(name):
        return sd[prefix + name].float()

    def q4(w):
        return Int4Weight.quantize(w.float(), gs)

    def bf(w):
        return w.to(torch.bfloat16).to(dev)

    model.cos_sin = rope_table(cfg, min(cfg.max_position, 1 << 16), rot=ROPE, device=dev)
    if model.has_embed:
        model.embed = bf(W("embed_tokens.weight"))
    model.layers = []
    for li in range(model.layer_start, model.layer_end):
        p = f"layers.{li}."
        a = p + "self_attn."
        qb = W(a + "q_b_proj.weight").view(hq, nope + ROPE, -1)
        qb = torch.cat([qb[:, :nope], qb[:, nope:][:, perm]], 1).reshape(hq * (nope + ROPE), -1)
        kva = W(a + "kv_a_proj_with_mqa.weight")
        kva = torch.cat([kva[:LATENT], kva[LATENT:][perm]])
        kva_q = q4(kva)
        kv_a = QLinear(type(kva_q).cat_rows([kva_q, Int4Pad.zeros(640 - ROW, H, gs, kva_q)]), dev)
        kvb = q4(W(a + "kv_b_proj.weight")).dequant_bf16().view(hq, nope + vd, LATENT)
        w_uk, w_uv = kvb[:, :nope].contiguous(), kvb[:, nope:].contiguous()
        if torch.device(dev).type == "cuda":
            w_uk, w_uv = w_uk.to(dev), w_uv.to(dev)
        else:
            w_uk, w_uv = w_uk.float(), w_uv.float()
        ind = None
        if cfg.layer_has_indexer(li):
            i = a + "indexer."
            ind = Indexer(wq_b=QLinear(q4(W(i + "wq_b.weight")), dev),
                          wk=QLinear(q4(W(i + "wk.weight")), dev),
                          k_norm_w=W(i + "k_norm.weight").to(dev),
                          k_norm_b=W(i + "k_norm.bias").to(dev),
                          w_proj=bf(W(i + "weights_proj.weight")))
        o = QLinear(q4(W(a + "o_proj.weight")), dev)
        attn = DSAAttention(q_a=QLinear(q4(W(a + "q_a_proj.weight")), dev),
                            q_a_norm=bf(W(a + "q_a_layernorm.weight")),
                            q_b=QLinear(q4(qb), dev), kv_a=kv_a,
                            kv_a_norm=bf(W(a + "kv_a_layernorm.weight")), w_uk=w_uk, w_uv=w_uv,
                            o=o, indexer=ind)
        m = p + "mlp."
        dense = router = bias = bank = shared = None
        if li < cfg.first_k_dense_replace:
            dense = (QLinear(q4(torch.cat([W(m + "gate_proj.weight"), W(m + "up_proj.weight")])),
                             dev, interleave_gate_up=True),
                     QLinear(q4(W(m + "down_proj.weight")), dev))
        else:
            router = bf(W(m + "gate.weight"))
            bias = W(m + "gate.e_score_correction_bias").to(dev)
            gu, dn = W(m + "experts.gate_up_proj"), W(m + "experts.down_proj")
            bank = ExpertBank([q4(gu[e]) for e in range(cfg.num_experts)],
                              [q4(dn[e]) for e in range(cfg.num_experts)], dev)
            se = m + "shared_experts."
            shared = (QLinear(q4(torch.cat([W(se + "gate_proj.weight"), W(se + "up_proj.weight")])),
                              dev, interleave_gate_up=True),
                      QLinear(q4(W(se + "down_proj.weight")), dev))
        model.layers.append(MoELayer(
            in_norm=bf(W(p + "input_layernorm.weight")),
            post_norm=bf(W(p + "post_attention_layernorm.weight")), qkv=attn, o=o, q_norm=None,
            k_norm=None, dense=dense, router=router, router_bias=bias, experts=bank, shared=shared))
    if model.has_head:
        model.final_norm = bf(W("norm.weight"))
        head = sd.get("lm_head.weight")
        model.lm_head = QLinear(q4((head if head is not None else
                                    sd[prefix + "embed_tokens.weight"]).float()), dev)
    return model


class GLM5MTP:
    """GLM-5's multi-token-prediction head (``num_nextn_predict_layers`` = 1,
    the DeepSeek-V3 MTP module stored as layer ``num_layers``), used as a
    speculative-decoding drafter.  Row j of the head reads the target's
    pre-norm hidden ``h_j`` at position j and the token at position j + 1, and
    predicts the token at j + 2::

        x  = rmsnorm(embed[t_{j+1}], enorm)
        h  = rmsnorm(final_norm(h_j), hnorm)   (chain steps: rmsnorm(h', hnorm))
        h' = block(eh_proj [x ; h])            one MLA + DSA + MoE decoder layer
        t_{j+2} = argmax lm_head(rmsnorm(h', shared_head.norm))

    (crates/cascadia-engine-sparse-moe/src/glm/mtp.rs:1-20 and :66-112 for
    the chain; ``embed``, ``final_norm`` and ``lm_head`` are the target's.)

    The reference clears the block's KV before each draft chain, so a draft
    attends only to the chain before it.  Here the block keeps a paged latent
    KV over the whole sequence: every verified position gets a row (its
    target hidden and the verified next token, one ragged forward per round
    for all sequences), and only the chain rows are rewound after the verify.
    ``eh_proj`` stays bf16 (the reference's notes: INT4 there collapses the
    acceptance rate); the block is INT4 like every other layer.
    """

    def __init__(self, target: GLM5Model):
        cfg = target.cfg
        assert cfg.num_nextn_predict_layers >= 1, "config has no MTP layer"
        self.target = target
        self.cfg = cfg
        self.device = target.device
        L = cfg.num_layers
        self.block = GLM5Model(cfg, target.device, layer_start=L, layer_end=L + 1,
                               has_embed=False, has_head=False)
        h = cfg.hidden_size
        ones = lambda: torch.ones(h, dtype=torch.bfloat16, device=self.device)  # noqa: E731
        self.enorm, self.hnorm, self.head_norm = ones(), ones(), ones()
        self.eh_proj = None

    @property
    def kv(self):
        return self.block.kv

    def init_random(self, seed: int = 0, std: float = 0.02, gen_device=None):
        from .llama import _layer_generator
        from .moe import BF16Linear

        self.block.init_random(seed, std, gen_device)
        h = self.cfg.hidden_size
        dev = torch.device(gen_device) if gen_device is not None else self.device
        g = _layer_generator(seed, 100002, dev)
        self.eh_proj = BF16Linear(torch.randn(h, 2 * h, generator=g, device=dev) * std,
                                  self.device)
        return self

    def allocate_kv(self, num_blocks: int):
        return self.block.allocate_kv(num_blocks)

    def step(self, batch: Batch, next_tokens: torch.Tensor, h_prev: torch.Tensor,
             from_target: bool):
        """One forward of the head over ``batch`` (rows at the positions of
        ``h_prev``).  Returns (h' [T, H] bf16, greedy drafts [T] int32)."""
        t = self.target
        T, H = h_prev.shape
        x = t.embed_tokens(next_tokens)
        xn = torch.empty_like(x)
        t._norm(x, self.enorm, xn)
        hn = torch.empty_like(h_prev)
        if from_target:
            t._norm(h_prev, t.final_norm, hn)
            h_prev = hn.clone()
        t._norm(h_prev, self.hnorm, hn)
        hx = self.eh_proj(torch.cat([xn, hn], dim=-1)).contiguous()
        self.block.forward(batch, hx)
        y = torch.empty_like(hx)
        t._norm(hx, self.head_norm, y)
        return hx, t.greedy(t.lm_head(y))


def load_mtp_weights(mtp: GLM5MTP, sd: Dict[str, torch.Tensor],
                     prefix: str = "model.") -> GLM5MTP:
    """Fill the MTP head from a ``glm_moe_dsa`` state dict: the block is
    ``layers.{num_layers}`` (loaded like any decoder layer), plus ``enorm``,
    ``hnorm``, ``eh_proj`` and ``shared_head.norm`` of that layer."""
    from .moe import BF16Linear

    p = f"{prefix}layers.{mtp.cfg.num_layers}."
    dev = mtp.device
    bf = lambda n: sd[p + n].to(torch.bfloat16).to(dev)  # noqa: E731
    load_hf_weights(mtp.block, sd, prefix)
    mtp.enorm, mtp.hnorm = bf("enorm.weight"), bf("hnorm.weight")
    mtp.head_norm = bf("shared_head.norm.weight")
    mtp.eh_proj = BF16Linear(sd[p + "eh_proj.weight"].float(), dev)
    return mtp
