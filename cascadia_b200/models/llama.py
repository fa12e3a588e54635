"""Llama-family INT4 decoder (dense), tensor- and pipeline-parallel aware.

One ``LlamaModel`` holds the layers ``[layer_start, layer_end)`` of one
pipeline stage, sharded ``tp_size`` ways:

* column-parallel: fused QKV (heads split), fused gate/up (interleaved per
  128-row tile so the GEMM epilogue applies SiLU(gate)*up);
* row-parallel: o_proj and down_proj, followed by a sum over the TP group
  (``TPGroup.all_reduce`` or one of the fused GEMM+collective paths);
* vocab-parallel LM head with a (value, index) argmax merge.

Math (per layer): pre-norm RMSNorm -> QKV -> RoPE (llama3 scaling) -> paged
GQA attention -> o_proj (+residual) -> RMSNorm -> SwiGLU -> down (+residual);
the same decoder the reference exports per stage
(tools/export_shards.py:657 cached_layer_forward_sdpa, :822-989 stage wrappers).

On CUDA every op is one of our sm_100a kernels; on CPU the forward uses the
fp32 oracle in ``ops.reference`` (the CPU engine / BASELINE CPU config).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List, Optional, Sequence

import torch

from .. import ops
from ..ops import reference as ref
from ..quant import Int4Weight
from ..runtime.kv_cache import BLOCK_SIZE, KVCache
from .config import ModelConfig, rope_table


# When set (model writers), every QLinear keeps its Int4Weight in `.int4`.
KEEP_INT4 = False


class QLinear:
    """An INT4 weight ready for its device: kernel blob on CUDA, fp32 on CPU."""

    def __init__(self, w: Int4Weight, device, interleave_gate_up: bool = False):
        self.n, self.k, self.group_size = w.n, w.k, w.group_size
        self.interleaved = interleave_gate_up
        self.int4 = w if KEEP_INT4 else None
        device = torch.device(device)
        if device.type == "cuda":
            self.blob = w.to(device).blob(interleave_gate_up)
            self.w_ref = None
        else:
            self.blob = None
            self.w_ref = w.dequant_bf16().float()  # exact kernel values, fp32 storage

    def __call__(self, x, epilogue=ops.EPI_STORE, residual=None, out=None):
        if self.blob is not None:
            return ops.w4a16_gemm(x, self.blob, self.n, self.group_size, epilogue, residual, out)
        y = x.float() @ self.w_ref.t()
        if epilogue == ops.EPI_SILU:
            y = ref.silu_mul(y[:, :self.n // 2], y[:, self.n // 2:])
        elif epilogue == ops.EPI_RESID:
            y = y + residual.float()
        y = y.to(torch.bfloat16)
        if out is not None:
            out.copy_(y)
            return out
        return y


@dataclass
class LayerWeights:
    in_norm: torch.Tensor
    post_norm: torch.Tensor
    qkv: QLinear
    o: QLinear
    gate_up: QLinear
    down: QLinear
    sparse: Optional[object] = None  # ops.ffn_sparse.SparseFFN when enabled


class TPGroup:
    """Tensor-parallel communicator used by the models.

    NCCL all-reduce is the baseline (and prefill) path; when ``fused`` is set
    (parallel.tp.FusedTP), decode-sized batches use the peer-memory
    all-reduce + RMSNorm kernel instead."""

    def __init__(self, rank: int = 0, size: int = 1, group=None):
        self.rank, self.size, self.group = rank, size, group
        self.fused = None

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        if self.size > 1:
            torch.distributed.all_reduce(x, group=self.group)
        return x

    def all_gather_rows(self, x: torch.Tensor) -> torch.Tensor:
        """[n, ...] on each rank -> [size, n, ...]."""
        if self.size == 1:
            return x.unsqueeze(0)
        out = torch.empty((self.size * x.shape[0],) + tuple(x.shape[1:]), dtype=x.dtype,
                          device=x.device)
        torch.distributed.all_gather_into_tensor(out, x.contiguous(), group=self.group)
        return out.view((self.size,) + tuple(x.shape))


def vocab_shard_rows(vocab_size: int, tp: int) -> int:
    """LM-head rows per rank at TP=`tp`: ceil(V / tp) rounded up to the
    GEMM's 128-row tile (e.g. 128256 -> 64128 / 32128 / 16128 at TP 2/4/8)."""
    if tp == 1:
        return vocab_size
    return -(-vocab_size // (tp * 128)) * 128


def _layer_generator(seed: int, layer: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed * 1000003 + layer * 7919 + 17)
    return g


def random_int4(n: int, k: int, g: torch.Generator, device, std=0.02, group_size=128,
                scale_dtype=torch.float16) -> Int4Weight:
    w = torch.randn(n, k, generator=g, device=device) * std
    return Int4Weight.quantize(w, group_size, scale_dtype)


class LlamaModel:
    def __init__(self, cfg: ModelConfig, device, tp: Optional[TPGroup] = None,
                 layer_start: int = 0, layer_end: Optional[int] = None,
                 has_embed: bool = True, has_head: bool = True):
        self.cfg = cfg
        self.device = torch.device(device)
        self.tp = tp or TPGroup()
        self.layer_start = layer_start
        self.layer_end = cfg.num_layers if layer_end is None else layer_end
        self.has_embed = has_embed
        self.has_head = has_head
        t = self.tp.size
        assert cfg.num_heads % t == 0 and cfg.num_kv_heads % t == 0, "heads must divide TP"
        self.hq = cfg.num_heads // t
        self.hkv = cfg.num_kv_heads // t
        self.d = cfg.head_dim
        self.inter = cfg.intermediate_size // t
        # Vocab-parallel LM head: every rank holds `vocab_shard` rows, a
        # multiple of 128 (the GEMM's row tile); rows at or past the true
        # vocabulary are zero padding that argmax and full_logits skip.
        self.vocab_shard = vocab_shard_rows(cfg.vocab_size, t)
        self.vocab_valid = max(0, min(self.vocab_shard,
                                      cfg.vocab_size - self.tp.rank * self.vocab_shard))
        self.layers: List[LayerWeights] = []
        self.embed: Optional[torch.Tensor] = None
        self.final_norm: Optional[torch.Tensor] = None
        self.lm_head: Optional[QLinear] = None
        self.cos_sin: Optional[torch.Tensor] = None
        self.kv: Optional[KVCache] = None
        self.scale = 1.0 / math.sqrt(self.d)

    @property
    def num_local_layers(self) -> int:
        return self.layer_end - self.layer_start

    # ------------------------------------------------------------ weights
    def init_random(self, seed: int = 0, std: float = 0.02, gen_device=None):
        """Random N(0, std) weights, INT4 sym group-quantised, generated per
        layer on the device with a layer-keyed seed so every TP/PP split of the
        same (seed, config) holds slices of the same full model."""
        cfg, t, r = self.cfg, self.tp.size, self.tp.rank
        # Generate where asked (CPU keeps CPU/GPU parity tests bit-identical),
        # then move every finished tensor to the model's device.
        dev = torch.device(gen_device) if gen_device is not None else self.device
        gs = cfg.group_size
        h, d = cfg.hidden_size, cfg.head_dim
        self.cos_sin = rope_table(cfg, min(cfg.max_position, 1 << 16), device=self.device)
        if self.has_embed or (self.has_head and cfg.tie_word_embeddings):
            g = _layer_generator(seed, 100000, dev)
            self.embed = (torch.randn(cfg.vocab_size, h, generator=g, device=dev) * std).to(
                torch.bfloat16).to(self.device)
        for li in range(self.layer_start, self.layer_end):
            g = _layer_generator(seed, li, dev)
            q = random_int4(cfg.num_heads * d, h, g, dev, std, gs)
            k = random_int4(cfg.num_kv_heads * d, h, g, dev, std, gs)
            v = random_int4(cfg.num_kv_heads * d, h, g, dev, std, gs)
            o = random_int4(h, cfg.num_heads * d, g, dev, std, gs)
            gate = random_int4(cfg.intermediate_size, h, g, dev, std, gs)
            up = random_int4(cfg.intermediate_size, h, g, dev, std, gs)
            down = random_int4(h, cfg.intermediate_size, g, dev, std, gs)
            self.layers.append(self._shard_layer(
                q, k, v, o, gate, up, down,
                torch.ones(h, dtype=torch.bfloat16, device=dev),
                torch.ones(h, dtype=torch.bfloat16, device=dev)))
            del q, k, v, o, gate, up, down
        if self.has_head:
            self.final_norm = torch.ones(h, dtype=torch.bfloat16, device=self.device)
            if cfg.tie_word_embeddings:
                head = Int4Weight.quantize(self.embed.to(dev).float(), gs)
            else:
                g = _layer_generator(seed, 100001, dev)
                head = random_int4(cfg.vocab_size, h, g, dev, std, gs)
            self.lm_head = QLinear(self._vocab_shard(head), self.device)
        return self

    def _vocab_shard(self, w: Int4Weight) -> Int4Weight:
        """This rank's `vocab_shard` LM-head rows; rows past the vocabulary
        are zero (nibble 8 with scale 0), so their logits are exactly 0 and
        the argmax never looks at them."""
        t, r = self.tp.size, self.tp.rank
        if t == 1:
            return w
        vs, valid = self.vocab_shard, self.vocab_valid
        part = w.rows(r * vs, r * vs + valid)
        if valid == vs:
            return part
        pad = vs - valid
        dev = w.packed.device
        zeros = Int4Weight(torch.full((pad, w.packed.shape[1]), -2004318072, dtype=torch.int32,
                                      device=dev),  # 0x88888888: eight nibbles of value 0
                           torch.zeros((pad, w.scales.shape[1]), dtype=w.scales.dtype, device=dev),
                           w.group_size)
        return Int4Weight.cat_rows([part, zeros]) if valid else zeros

    def _shard_layer(self, q, k, v, o, gate, up, down, in_norm, post_norm) -> LayerWeights:
        t, r, d = self.tp.size, self.tp.rank, self.cfg.head_dim
        hq, hkv, it = self.hq, self.hkv, self.inter
        qkv = Int4Weight.cat_rows([q.rows(r * hq * d, (r + 1) * hq * d),
                                   k.rows(r * hkv * d, (r + 1) * hkv * d),
                                   v.rows(r * hkv * d, (r + 1) * hkv * d)])
        gu = Int4Weight.cat_rows([gate.rows(r * it, (r + 1) * it), up.rows(r * it, (r + 1) * it)])
        dev = self.device
        return LayerWeights(
            in_norm=in_norm.to(dev), post_norm=post_norm.to(dev),
            qkv=QLinear(qkv, dev),
            o=QLinear(o.cols(r * hq * d, (r + 1) * hq * d), dev),
            gate_up=QLinear(gu, dev, interleave_gate_up=True),
            down=QLinear(down.cols(r * it, (r + 1) * it), dev))

    def load_layer(self, li: int, tensors: dict, group_size: int):
        """Install one layer from a shard's tensors (canonical INT4 form)."""
        def w(name):
            return Int4Weight(tensors[name + ".packed"], tensors[name + ".scales"], group_size)
        self.layers.append(self._shard_layer(
            w("q_proj"), w("k_proj"), w("v_proj"), w("o_proj"), w("gate_proj"), w("up_proj"),
            w("down_proj"), tensors["input_layernorm"].to(torch.bfloat16),
            tensors["post_attention_layernorm"].to(torch.bfloat16)))

    # ------------------------------------------------------------ KV cache
    def enable_ffn_sparsity(self, tau_all: float = 0.05, taus=None):
        """Single-token steps (TP=1) run the activation-sparse FFN: lanes with
        |silu(gate)| below tau (x the token's max) skip up and down.  Off by
        default; needs the INT4 weights kept at build time (KEEP_INT4)."""
        from ..ops.ffn_sparse import SparseFFN

        for i, lw in enumerate(self.layers):
            gu, dn = lw.gate_up.int4, lw.down.int4
            if gu is None or dn is None:
                raise RuntimeError("build the model with llama.KEEP_INT4 = True first")
            inter = gu.n // 2
            lw.sparse = SparseFFN(gu.rows(0, inter), gu.rows(inter, 2 * inter), dn, self.device,
                                  tau_all, taus[i] if taus is not None else None)

    def early_exit(self, num_layers: int) -> "LlamaModel":
        """A model that shares this one's embedding, first ``num_layers``
        layers, final norm and LM head (no weight copies) and has its own KV
        cache: the draft of self-speculative decoding by early exit
        (LayerSkip, Elhoushi et al. 2024).  Single GPU, whole model only."""
        assert self.tp.size == 1 and self.layer_start == 0 and self.has_embed and self.has_head
        assert 0 < num_layers <= len(self.layers)
        import copy

        cfg = copy.copy(self.cfg)
        cfg.num_layers = num_layers
        d = LlamaModel(cfg, self.device)
        d.cos_sin = self.cos_sin
        d.embed = self.embed
        d.layers = self.layers[:num_layers]
        d.final_norm = self.final_norm
        d.lm_head = self.lm_head
        return d

    # ------------------------------------------------ pipeline stage payload
    # What one stage hands the next per token row.  For most families it is
    # the hidden row itself; a family whose later layers need more (Gemma-4:
    # per-layer inputs and the K/V rows of shared-cache source layers)
    # widens it.
    @property
    def payload_in_width(self) -> int:
        return self.cfg.hidden_size

    @property
    def payload_out_width(self) -> int:
        return self.cfg.hidden_size

    def pack_payload(self, hidden: torch.Tensor, batch: "Batch") -> torch.Tensor:
        return hidden

    def unpack_payload(self, buf: torch.Tensor, batch: "Batch",
                       out: Optional[torch.Tensor] = None) -> torch.Tensor:
        if out is None:
            return buf
        out.copy_(buf)
        return out

    def allocate_kv(self, num_blocks: int) -> KVCache:
        self.kv = KVCache(self.num_local_layers, num_blocks, self.hkv, self.d, self.device)
        return self.kv

    def kv_bytes_per_block(self) -> int:
        return KVCache.bytes_per_block(self.num_local_layers, self.hkv, self.d)

    # ------------------------------------------------------------ forward
    def embed_tokens(self, ids: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        if out is None:
            out = torch.empty(ids.shape[0], self.cfg.hidden_size, dtype=torch.bfloat16,
                              device=self.device)
        if self.device.type == "cuda":
            ops.embedding(ids, self.embed, out)
        else:
            out.copy_(self.embed[ids.long()])
        return out

    def _norm(self, x, w, out, residual=None):
        if self.device.type == "cuda":
            return ops.rmsnorm(x, w, out, self.cfg.rms_eps, residual=residual)
        if residual is not None:
            residual.copy_((x.float() + residual.float()).to(torch.bfloat16))
            x = residual
        out.copy_(ref.rmsnorm(x, w, self.cfg.rms_eps).to(torch.bfloat16))
        return out

    def forward(self, batch: "Batch", hidden: torch.Tensor) -> torch.Tensor:
        """Run this stage's layers on `hidden` ([T, H] bf16, the residual
        stream) in place; returns the residual stream (pre final-norm)."""
        cfg = self.cfg
        T = hidden.shape[0]
        h = torch.empty_like(hidden)
        fz = self.tp.fused
        if fz is not None and self.device.type == "cuda" and T <= fz.max_tokens:
            return self._forward_fused(batch, hidden, h, fz)
        pending: Optional[torch.Tensor] = None  # TP partial sum not yet added
        tp1 = self.tp.size == 1
        for i, lw in enumerate(self.layers):
            self._norm(pending if pending is not None else hidden, lw.in_norm, h,
                       residual=hidden if pending is not None else None)
            attn = self._qkv_attention(i, lw, h, batch)
            if tp1:
                lw.o(attn, ops.EPI_RESID, residual=hidden, out=hidden)
                self._norm(hidden, lw.post_norm, h)
            else:
                part = self.tp.all_reduce(lw.o(attn))
                self._norm(part, lw.post_norm, h, residual=hidden)
            if tp1 and T == 1 and lw.sparse is not None:
                lw.sparse(h, residual=hidden, out=hidden)  # activation-sparse FFN
                pending = None
                continue
            act = lw.gate_up(h, ops.EPI_SILU)
            if tp1:
                lw.down(act, ops.EPI_RESID, residual=hidden, out=hidden)
                pending = None
            else:
                pending = self.tp.all_reduce(lw.down(act))
        if pending is not None:
            hidden.copy_((hidden.float() + pending.float()).to(torch.bfloat16)) \
                if self.device.type != "cuda" else hidden.add_(pending)
        return hidden

    def _forward_fused(self, batch, hidden, h, fz):
        """TP forward with the peer-memory all-reduce fused into RMSNorm: the
        row-parallel GEMMs write partials into the symmetric buffer; each
        all-reduce also applies the next norm (post-attention norm after
        o_proj, the next layer's input norm after down_proj)."""
        T = hidden.shape[0]
        eps = self.cfg.rms_eps
        self._norm(hidden, self.layers[0].in_norm, h)
        for i, lw in enumerate(self.layers):
            attn = self._qkv_attention(i, lw, h, batch)
            nxt = self.layers[i + 1].in_norm if i + 1 < len(self.layers) else None
            if fz.push:
                # The GEMM delivers its partial into every rank's slots.
                fz.gemm_push(lw.o, attn, 0)
                fz.allreduce_pushed(0, T, hidden, lw.post_norm, h, eps)
                act = lw.gate_up(h, ops.EPI_SILU)
                fz.gemm_push(lw.down, act, 1)
                fz.allreduce_pushed(1, T, hidden, nxt, h, eps)
                continue
            lw.o(attn, out=fz.partial_out(0, T))
            fz.allreduce(0, T, hidden, lw.post_norm, h, eps)
            act = lw.gate_up(h, ops.EPI_SILU)
            lw.down(act, out=fz.partial_out(1, T))
            fz.allreduce(1, T, hidden, nxt, h if nxt is not None else h, eps)
        return hidden

    def _qkv_attention(self, li: int, lw: LayerWeights, h: torch.Tensor, batch: "Batch"):
        """q/k/v projection + attention.  On the GPU, when the shapes allow,
        the projection's epilogue applies RoPE and writes K / V into the
        paged cache (one launch less per layer)."""
        T = h.shape[0]
        if (self.device.type == "cuda" and lw.qkv.blob is not None and
                ops.rope_fusable(T, self.d, self.cfg.rot_dim, lw.qkv.group_size)):
            qkv = torch.empty(T, lw.qkv.n, dtype=torch.bfloat16, device=self.device)
            ops.w4a16_gemm_rope_kv(h, lw.qkv.blob, lw.qkv.n, lw.qkv.group_size, qkv,
                                   batch.positions, self.cos_sin, batch.slots, self.kv.k,
                                   self.kv.v, li, self.hq, self.hkv)
            return self._attention(li, qkv, batch, roped=True)
        return self._attention(li, lw.qkv(h), batch)

    def _attention(self, li: int, qkv: torch.Tensor, batch: "Batch",
                   roped: bool = False) -> torch.Tensor:
        hq, hkv, d = self.hq, self.hkv, self.d
        kv = self.kv
        T = qkv.shape[0]
        if self.device.type == "cuda":
            if not roped:
                ops.rope_kv_write(qkv, batch.positions, self.cos_sin, batch.slots, kv.k, kv.v,
                                  li, hq, hkv, d, self.cfg.rot_dim)
            out = torch.empty(T, hq * d, dtype=torch.bfloat16, device=self.device)
            q = qkv[:, :hq * d]
            win, sinks = self.cfg.sliding_window, self.cfg.attention_sinks
            if batch.is_decode:
                ops.attn_decode(q, kv.k, kv.v, batch.block_tables, batch.seq_lens, out, li,
                                batch.num_splits, batch.blocks_per_split, batch.part_o,
                                batch.part_ml, self.scale, win, sinks)
            else:
                ops.attn_prefill(q, kv.k, kv.v, batch.block_tables, batch.tiles, out, li,
                                 self.scale, win, sinks)
            return out
        # CPU oracle path.
        x = qkv.float().view(T, hq + 2 * hkv, d)
        pos = batch.positions.long()
        q = ref.apply_rope(x[:, :hq], pos, self.cos_sin, self.cfg.rot_dim)
        k = ref.apply_rope(x[:, hq:hq + hkv], pos, self.cos_sin, self.cfg.rot_dim)
        v = x[:, hq + hkv:]
        slots = batch.slots.long()
        valid = slots >= 0
        sb, so = slots[valid] // BLOCK_SIZE, slots[valid] % BLOCK_SIZE
        kv.k[li, sb, :, so] = k[valid].to(torch.bfloat16)
        kv.v[li, sb, :, so] = v[valid].to(torch.bfloat16)
        out = torch.empty(T, hq * d, dtype=torch.float32)
        row = 0
        for sid, ql in zip(batch.seq_ids, batch.q_lens):
            kk, vv = kv.gather(li, sid)
            ctx = int(batch.ctx_len_of(sid))
            o = ref.attention(q[row:row + ql], kk[:ctx], vv[:ctx], pos[row:row + ql], self.scale,
                              self.cfg.sliding_window, self.cfg.attention_sinks)
            out[row:row + ql] = o.reshape(ql, hq * d)
            row += ql
        return out.to(torch.bfloat16)

    def head(self, hidden_last: torch.Tensor) -> torch.Tensor:
        """Final norm + (vocab-sharded) LM head: bf16 logits [B, V/tp]."""
        h = torch.empty_like(hidden_last)
        self._norm(hidden_last, self.final_norm, h)
        return self.lm_head(h)

    def greedy(self, logits: torch.Tensor) -> torch.Tensor:
        """Argmax over the full vocabulary (merging vocab shards)."""
        B = logits.shape[0]
        if self.device.type != "cuda":
            return ref.argmax(self.full_logits(logits))
        idx = torch.empty(B, dtype=torch.int32, device=self.device)
        if self.tp.size == 1:
            return ops.argmax(logits, idx)
        val = torch.empty(B, dtype=torch.float32, device=self.device)
        # Only the real vocabulary rows of this shard (a view with the same
        # row stride): padded rows are never candidates.
        ops.argmax(logits[:, :self.vocab_valid], idx, val,
                   idx_offset=self.tp.rank * self.vocab_shard)
        pair = torch.stack([val, idx.float()], dim=1)  # exact for idx < 2^24
        allp = self.tp.all_gather_rows(pair)  # [tp, B, 2]
        best = torch.argmax(allp[:, :, 0], dim=0)  # first (lowest rank) wins ties
        return allp[best, torch.arange(B, device=self.device), 1].to(torch.int32)

    def full_logits(self, logits: torch.Tensor) -> torch.Tensor:
        """[B, vocab_size] logits from every rank's (padded) shard."""
        if self.tp.size == 1:
            return logits
        allp = self.tp.all_gather_rows(logits.contiguous())  # [tp, B, vocab_shard]
        full = allp.permute(1, 0, 2).reshape(logits.shape[0], -1)
        return full[:, :self.cfg.vocab_size]


@dataclass
class Batch:
    """Inputs of one forward of a stage (prefill or decode)."""
    seq_ids: List[str]
    q_lens: List[int]
    ctx_lens: List[int]           # total context after this step, per sequence
    positions: torch.Tensor       # int32 [T]
    slots: torch.Tensor           # int32 [T]
    block_tables: torch.Tensor    # int32 [B, W]
    seq_lens: torch.Tensor        # int32 [B] (= ctx_lens on device)
    is_decode: bool
    tiles: Optional[torch.Tensor] = None
    num_splits: int = 1
    blocks_per_split: int = 1
    part_o: Optional[torch.Tensor] = None
    part_ml: Optional[torch.Tensor] = None

    def ctx_len_of(self, sid: str) -> int:
        return self.ctx_lens[self.seq_ids.index(sid)]

    @property
    def last_rows(self) -> List[int]:
        out, r = [], 0
        for ql in self.q_lens:
            r += ql
            out.append(r - 1)
        return out


def build_batch(model: LlamaModel, seq_ids: Sequence[str], q_lens: Sequence[int],
                positions_start: Sequence[int], decode: bool, device=None,
                width: Optional[int] = None) -> Batch:
    """Reserve KV for the new tokens and build the device inputs."""
    kv = model.kv
    device = device or model.device
    pos, slots, ctx = [], [], []
    for sid, ql, p0 in zip(seq_ids, q_lens, positions_start):
        kv.reserve(sid, p0 + ql)
        kv.slide(sid, model.cfg, p0)
        s = kv.seqs[sid]
        s.length = max(s.length, p0 + ql)
        pos.extend(range(p0, p0 + ql))
        slots.extend(s.slots(p0, p0 + ql))
        ctx.append(p0 + ql)
    maxb = max((len(kv.seqs[s].blocks) for s in seq_ids), default=1)
    width = max(width or 0, maxb)
    b = Batch(seq_ids=list(seq_ids), q_lens=list(q_lens), ctx_lens=ctx,
              positions=torch.tensor(pos, dtype=torch.int32).to(device),
              slots=torch.tensor(slots, dtype=torch.int32).to(device),
              block_tables=kv.block_table(list(seq_ids), width, device),
              seq_lens=torch.tensor(ctx, dtype=torch.int32).to(device), is_decode=decode)
    if torch.device(device).type == "cuda":
        if decode:
            b.num_splits, b.blocks_per_split = ops.decode_split_plan(len(seq_ids), model.hkv, maxb)
            g = model.hq // model.hkv
            n = len(seq_ids) * model.hkv * b.num_splits * g
            b.part_o = torch.empty(n * model.d, dtype=torch.float32, device=device)
            b.part_ml = torch.empty(n * 2, dtype=torch.float32, device=device)
        else:
            b.tiles = ops.prefill_tiles(q_lens, ctx, device)
    return b
