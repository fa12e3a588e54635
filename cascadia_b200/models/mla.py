"""Kimi-K2 / DeepSeek-V3-shaped model: multi-head latent attention (MLA)
followed by the sparse-MoE FFN of :mod:`.moe` (first layers dense, sigmoid
routing with bias, one shared expert).

Attention per layer (reference: crates/cascadia-int4-gemm/src/shell.rs:81-341):

    q   = q_b(rmsnorm(q_a(x)))                  [T, heads, nope 128 | rope 64]
    kva = kv_a(x)                               [T, latent 512 | rope 64]
    c   = rmsnorm(kva[:, :512]);  k_rope = rope(kva[:, 512:])   (shared by heads)
    k_nope[h] = W_UK[h] c,  v[h] = W_UV[h] c    (kv_b rows of head h)
    o = o_proj(concat_h softmax(q[h] . k[h] / sqrt(192)) v[h])

The CPU oracle computes exactly that (expanded K/V).  The GPU path runs the
absorbed form: the paged cache keeps one 576-wide row [c | k_rope] per token
(csrc/mla.cu), queries are absorbed into the latent space
(q_lat[h] = W_UK[h]^T q_nope[h]) and the latent output is expanded once
(o[h] = W_UV[h] o_lat[h]); the absorptions are batched bf16 GEMMs.  Prefill
runs the same kernel with one virtual sequence per query token (causal by
its own context length).  RoPE rotates interleaved pairs (x[2i], x[2i+1]),
which gives the same scores as the reference's de-interleave + rotate-half.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import numpy as np
import torch

from .. import ops
from ..ops import reference as ref
from ..runtime.kv_cache import BLOCK_SIZE, KVCache
from .config import rope_table
from .llama import Batch, QLinear, random_int4
from .moe import MoEModel

LATENT = 512
ROPE = 64
ROW = LATENT + ROPE


class LatentKVCache(KVCache):
    """Paged latent cache: [layers, blocks, 16, 576] (no separate V pool).
    On GPU the rows of a block are chunk-swizzled by the writing kernel."""

    def __init__(self, num_layers: int, num_blocks: int, device):
        from ..runtime.kv_cache import BlockAllocator

        self.num_layers = num_layers
        self.num_blocks = num_blocks
        self.kv_heads = 1
        self.head_dim = ROW
        self.k = torch.zeros(num_layers, num_blocks, BLOCK_SIZE, ROW, dtype=torch.bfloat16,
                             device=device)
        self.v = None
        self.allocator = BlockAllocator(num_blocks)
        self.seqs = {}

    @staticmethod
    def bytes_per_block(num_layers, *_args, **_kw) -> int:
        return num_layers * BLOCK_SIZE * ROW * 2

    def gather_latent(self, layer: int, seq_id: str) -> torch.Tensor:
        """Dense [len, 576] rows of one sequence (CPU layout, unswizzled)."""
        s = self.seqs[seq_id]
        ids = torch.tensor(s.blocks, dtype=torch.long, device=self.k.device)
        return self.k[layer, ids].reshape(-1, ROW)


@dataclass
class MLAAttention:
    q_a: Optional[QLinear]          # [q_lora, H] (None: q_b takes x directly)
    q_a_norm: Optional[torch.Tensor]
    q_b: QLinear                    # [heads * 192, q_lora or H]
    kv_a: QLinear                   # [576 padded to 640, H]
    kv_a_norm: torch.Tensor         # [512]
    w_uk: torch.Tensor              # [heads, 128, 512] bf16 (fp32 on CPU)
    w_uv: torch.Tensor              # [heads, 128, 512]
    o: QLinear                      # [H, heads * 128]


class MLAModel(MoEModel):
    def __init__(self, cfg, device, **kw):
        kw.setdefault("bf16_attention", False)
        super().__init__(cfg, device, **kw)
        assert cfg.kv_lora_rank == LATENT and cfg.qk_rope_head_dim == ROPE, \
            "the MLA kernels are built for a 512-wide latent and a 64-wide rope key"
        self.nope = cfg.qk_nope_head_dim   # 128 (Kimi-K2) or 192 (GLM-5)
        self.vd = cfg.v_head_dim           # 128 or 256
        self.qk_dim = self.nope + ROPE
        # The q_a / kv_a RMSNorms use eps 1e-6 (the published MLA norms).
        self.lora_eps = 1e-6
        self.scale = 1.0 / math.sqrt(self.qk_dim)
        self.hq = cfg.num_heads

    # ------------------------------------------------------------ weights
    def init_random(self, seed: int = 0, std: float = 0.02, gen_device=None):
        super().init_random(seed, std, gen_device)
        self.cos_sin = rope_table(self.cfg, min(self.cfg.max_position, 1 << 16), rot=ROPE,
                                  device=self.device)
        return self

    def _init_attention(self, g, dev, std):
        cfg = self.cfg
        h, gs, H = cfg.hidden_size, cfg.group_size, cfg.num_heads
        q_a = q_a_norm = None
        if cfg.q_lora_rank:
            q_a = QLinear(random_int4(cfg.q_lora_rank, h, g, dev, std, gs), self.device)
            q_a_norm = torch.ones(cfg.q_lora_rank, dtype=torch.bfloat16, device=self.device)
            q_in = cfg.q_lora_rank
        else:
            q_in = h
        q_b = QLinear(random_int4(H * (cfg.qk_nope_head_dim + ROPE), q_in, g, dev, std, gs),
                      self.device)
        kva_w = random_int4(ROW, h, g, dev, std, gs)
        # Pad the 576 rows to 640 (the GEMM tiles 128 rows); pad rows are zero.
        pad = Int4Pad.zeros(640 - ROW, h, gs, kva_w)
        kv_a = QLinear(type(kva_w).cat_rows([kva_w, pad]), self.device)
        kv_b = random_int4(H * (cfg.qk_nope_head_dim + cfg.v_head_dim), LATENT, g, dev, std, gs)
        wb = kv_b.dequant_bf16().view(H, cfg.qk_nope_head_dim + cfg.v_head_dim, LATENT)
        w_uk = wb[:, :cfg.qk_nope_head_dim].contiguous()
        w_uv = wb[:, cfg.qk_nope_head_dim:].contiguous()
        if torch.device(self.device).type == "cuda":
            w_uk, w_uv = w_uk.to(self.device), w_uv.to(self.device)
        else:
            w_uk, w_uv = w_uk.float(), w_uv.float()
        o = QLinear(random_int4(h, H * cfg.v_head_dim, g, dev, std, gs), self.device)
        attn = MLAAttention(q_a=q_a, q_a_norm=q_a_norm, q_b=q_b, kv_a=kv_a,
                            kv_a_norm=torch.ones(LATENT, dtype=torch.bfloat16, device=self.device),
                            w_uk=w_uk, w_uv=w_uv, o=o)
        return attn, o

    def allocate_kv(self, num_blocks: int) -> KVCache:
        self.kv = LatentKVCache(self.num_local_layers, num_blocks, self.device)
        return self.kv

    def kv_bytes_per_block(self) -> int:
        return LatentKVCache.bytes_per_block(self.num_local_layers)

    # ------------------------------------------------------------ forward
    def forward(self, batch: Batch, hidden: torch.Tensor) -> torch.Tensor:
        h = torch.empty_like(hidden)
        for i, lw in enumerate(self.layers):
            self._norm(hidden, lw.in_norm, h)
            attn = self._mla(i, lw.qkv, h, batch)
            lw.o(attn, ops.EPI_RESID, residual=hidden, out=hidden)
            self._norm(hidden, lw.post_norm, h)
            if lw.dense is not None:
                act = lw.dense[0](h, ops.EPI_SILU)
                lw.dense[1](act, ops.EPI_RESID, residual=hidden, out=hidden)
            else:
                self._moe(lw, h, hidden)
        return hidden

    def _norm_eps(self, x, w, out, eps):
        if self.device.type == "cuda":
            return ops.rmsnorm(x, w, out, eps)
        out.copy_(ref.rmsnorm(x, w, eps).to(torch.bfloat16))
        return out

    def _q_and_kv(self, a: MLAAttention, x: torch.Tensor):
        """(q, normalised latent c, rope key, q_a residual or None)."""
        qa_n = None
        if a.q_a is not None:
            qa = a.q_a(x)
            qa_n = torch.empty_like(qa)
            self._norm_eps(qa, a.q_a_norm, qa_n, self.lora_eps)
            q = a.q_b(qa_n)
        else:
            q = a.q_b(x)
        kva = a.kv_a(x)  # [T, 640]: latent | rope key | zero pad
        c = torch.empty(x.shape[0], LATENT, dtype=x.dtype, device=x.device)
        self._norm_eps(kva[:, :LATENT], a.kv_a_norm, c, self.lora_eps)
        return q, c, kva[:, LATENT:ROW], qa_n

    def _mla(self, li: int, a: MLAAttention, x: torch.Tensor, batch: Batch) -> torch.Tensor:
        q, c, kr, _ = self._q_and_kv(a, x)
        if self.device.type == "cuda":
            return self._mla_gpu(li, a, q, c, kr, batch)
        return self._mla_cpu(li, a, q, c, kr, batch)

    def _virtual_seqs(self, batch: Batch):
        """Block tables and lengths with one row per query token (prefill:
        each token is a sequence of its own context length)."""
        if batch.is_decode:
            return batch.block_tables, batch.seq_lens
        return batch.block_tables.index_select(0, self._tok2seq(batch)), batch.positions + 1

    # ------------------------------------------------------------ GPU (absorbed)
    def _mla_gpu(self, li, a, q, c, kr, batch, sel=None):
        """sel: optional DSA selection (scores [T, ld] fp32, thresholds [T])."""
        T, H = q.shape[0], self.hq
        q3 = q.view(T, H, self.qk_dim)
        q_full = torch.empty(T, H, ROW, dtype=torch.bfloat16, device=q.device)
        # q_lat[t, h] = W_UK[h]^T q_nope[t, h]: one batched GEMM over heads.
        q_lat = torch.bmm(q3[:, :, :self.nope].transpose(0, 1), a.w_uk)  # [H, T, 512]
        q_full[:, :, :LATENT].copy_(q_lat.transpose(0, 1))
        ops.ext().mla_rope_write(c, kr, q3[:, 0, self.nope:], self.qk_dim, q_full,
                                 batch.positions, self.cos_sin, batch.slots, self.kv.k, li, H)
        o_lat = torch.empty(T, H, LATENT, dtype=torch.bfloat16, device=q.device)
        bt, lens = self._virtual_seqs(batch)
        splits, bps = mla_split_plan(T, H, bt.shape[1])
        part_o = part_ml = o_lat
        if splits > 1:
            part_o = torch.empty(T * H * splits * LATENT, dtype=torch.float32, device=q.device)
            part_ml = torch.empty(T * H * splits * 2, dtype=torch.float32, device=q.device)
        ops.ext().mla_decode(q_full, self.kv.k, bt, lens, o_lat, li, splits, bps, part_o, part_ml,
                             self.scale, ops.status_buffer(q.device),
                             sel[0] if sel is not None else None,
                             sel[1] if sel is not None else None)
        ops.LAUNCHES.add(3 if splits > 1 else 2)
        out = torch.bmm(o_lat.transpose(0, 1), a.w_uv.transpose(1, 2))  # [H, T, v]
        return out.transpose(0, 1).reshape(T, H * self.vd)

    def _tok2seq(self, batch: Batch) -> torch.Tensor:
        key = tuple(batch.q_lens)
        cache = getattr(batch, "_tok2seq", None)
        if cache is None or cache[0] != key:
            idx = np.repeat(np.arange(len(batch.q_lens)), batch.q_lens)
            batch._tok2seq = (key, torch.from_numpy(idx).to(self.device))
        return batch._tok2seq[1]

    # ------------------------------------------------------------ CPU oracle
    def _mla_cpu(self, li, a, q, c, kr, batch, sel=None):
        T, H = q.shape[0], self.hq
        pos = batch.positions.long()
        q3 = q.float().view(T, H, self.qk_dim)
        q_rope = rope_pairs(q3[:, :, self.nope:], pos, self.cos_sin)
        k_rope = rope_pairs(kr.float().view(T, 1, ROPE), pos, self.cos_sin)[:, 0]
        rows = torch.cat([c.float(), k_rope], dim=1).to(torch.bfloat16)
        slots = batch.slots.long()
        valid = slots >= 0
        self.kv.k[li, slots[valid] // BLOCK_SIZE, slots[valid] % BLOCK_SIZE] = rows[valid]
        out = torch.empty(T, H, self.vd)
        r = 0
        for sid, ql in zip(batch.seq_ids, batch.q_lens):
            lat = self.kv.gather_latent(li, sid).float()
            ctx = int(batch.ctx_len_of(sid))
            cc, kk_r = lat[:ctx, :LATENT], lat[:ctx, LATENT:]
            k_nope = torch.einsum("hdl,tl->thd", a.w_uk, cc)          # [ctx, H, nope]
            v = torch.einsum("hdl,tl->thd", a.w_uv, cc)               # [ctx, H, v]
            k = torch.cat([k_nope, kk_r[:, None, :].expand(ctx, H, ROPE)], dim=2)
            qq = torch.cat([q3[r:r + ql, :, :self.nope], q_rope[r:r + ql]], dim=2)
            s = torch.einsum("qhd,thd->hqt", qq, k) * self.scale
            qpos = pos[r:r + ql]
            mask = torch.arange(ctx)[None, :] > qpos[:, None]
            if sel is not None:  # DSA: only the selected positions
                sc, thr = sel
                mask = mask | (sc[r:r + ql, :ctx] < thr[r:r + ql, None])
            s = s.masked_fill(mask[None], float("-inf"))
            p = torch.softmax(s, dim=-1)
            out[r:r + ql] = torch.einsum("hqt,thd->qhd", p, v)
            r += ql
        return out.reshape(T, H * self.vd).to(torch.bfloat16)


def rope_pairs(x: torch.Tensor, pos: torch.Tensor, cos_sin: torch.Tensor) -> torch.Tensor:
    """Rotate interleaved pairs (x[2i], x[2i+1]) by the angle of frequency i."""
    half = ROPE // 2
    cs = cos_sin[pos].float()
    cos, sin = cs[:, None, :half], cs[:, None, half:]
    x0, x1 = x[..., 0::2], x[..., 1::2]
    y = torch.empty_like(x)
    y[..., 0::2] = x0 * cos - x1 * sin
    y[..., 1::2] = x1 * cos + x0 * sin
    return y


def mla_split_plan(B: int, heads: int, width_blocks: int, sms: int = 148):
    """Context splits: double while the grid (head groups x sequences x
    splits) stays within ~4.6 waves of 3 CTAs per SM and every split keeps
    at least 16 blocks (256 tokens).  Fitted to graph-timed sweeps on B200
    (64 heads, 4096 tokens: batch 16 best at 16 splits, 97 us; batch 64 at
    8 splits, 292 us against 359 us unsplit)."""
    ctas = ((heads + 15) // 16) * B
    cap = max(3 * sms, 2048 * sms // 148)
    splits = 1
    while (ctas * splits * 2 <= cap and width_blocks // (splits * 2) >= 16
           and splits < 64):
        splits *= 2
    bps = -(-width_blocks // splits)
    return splits, bps


class Int4Pad:
    @staticmethod
    def zeros(n, k, gs, like):
        """INT4 rows that dequantise to exactly zero (nibble 8, scale 1)."""
        packed = torch.full((n, k // 8), 0x88888888 - (1 << 32), dtype=torch.int32,
                            device=like.packed.device)
        scales = torch.ones(n, k // gs, dtype=like.scales.dtype, device=like.scales.device)
        return type(like)(packed, scales, gs)
