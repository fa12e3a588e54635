"""DeepSeek-V4 (``deepseek_v4``) text model.

Architecture (the behaviour of the reference's Rust shell,
crates/cascadia-engine-sparse-moe/src/dsv4/{model,hc,attn_layer,compress,
indexer,rope,math}.rs, which follows DeepSeek's published inference code):

* **Hyper-Connections.** The residual stream is ``hc`` copies of the hidden
  vector per token.  Before every sublayer the flattened copies give
  ``(2 + hc) * hc`` mixing logits (a linear map scaled by the copies' inverse
  RMS); ``pre`` (sigmoid) weights reduce the copies to the sublayer input,
  ``post`` (2 x sigmoid) scales the sublayer output into each new copy, and
  ``comb`` (row softmax, then Sinkhorn row / column normalisation) mixes the
  old copies into the new ones (hc_split_sinkhorn, hc.rs:26).
* **Attention.** Low-rank q (``wq_a`` -> RMSNorm -> ``wq_b``, per-head plain
  RMS normalisation), ONE shared KV latent per token (MQA: the row is both
  K and V), RoPE on the last ``rope_head_dim`` dims as adjacent pairs,
  FP8 (e4m3, power-of-two block scales) quant-dequant of the non-rope
  channels, per-head attention sinks (a logit in the softmax denominator
  only), inverse RoPE on the output, grouped low-rank output projection.
  Each query sees a sliding window of raw latents plus compressed rows.
* **KV compression.** Layers with ratio r > 0 pool every r tokens into one
  row with a learned per-channel softmax gate (``wkv``, ``wgate``, ``ape``);
  ratio 4 overlaps windows (each block also pools the previous block's
  first-half channels).  Rows are RMS-normed, roped at the block's first
  position and FP8-simulated (compress.rs:33-268).
* **Indexer** (ratio-4 layers): its own rotate-variant compressor (Hadamard
  + FP4 e2m1 quant-dequant), index heads scored with ReLU and learned head
  weights pick ``index_topk`` compressed rows per query (indexer.rs).
  Ratio-16 layers attend to every compressed row.
* **MoE.** ``sqrt(softplus(logits))`` scores; the first ``n_hash_layers``
  route by a token-id -> expert table, the others by score + bias top-k;
  weights renormalised times ``route_scale``; SwiGLU experts with clamped
  gate / up (``swiglu_limit``) plus a shared expert (model.rs:215-240).
* **Head.** HC reduction with sigmoid weights, RMSNorm, fp32 logits.

Numerics follow the reference's dtype boundaries: activations are bf16
values held in fp32, every linear with bf16 weights rounds its fp32 result
to bf16, norms / ropes / mixes round where the reference does, and the
compressor / gate / HC logits stay fp32.

This implementation is batched over positions (prefill: every projection,
the compressor pooling, the indexer scores and the sparse attention run as
tensor ops over all tokens at once; on CUDA the HC pre-mix (RMS, mixing logits, Sinkhorn, reduction) is
our ``hc_pre`` kernel) with per-sequence decode state (raw-latent ring,
compressor windows, compressed caches).  The tiny exported model of the
reference (4 layers, hidden 64) and its recorded logits are the test
fixture.
"""
from __future__ import annotations

import json
import math
import os
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence

import numpy as np
import torch


# ------------------------------------------------------------------ numerics

def bf16r(t: torch.Tensor) -> torch.Tensor:
    """Round to the nearest bf16 value (kept in fp32)."""
    return t.to(torch.bfloat16).to(torch.float32)


def pow2_ceil(x: torch.Tensor) -> torch.Tensor:
    """2 ** ceil(log2(x)) for positive normal x, exact (from the exponent
    and mantissa bits)."""
    bits = x.to(torch.float32).view(torch.int32)
    exp = (bits >> 23) & 0xFF
    man = bits & 0x7FFFFF
    e = exp + (man != 0).to(torch.int32)
    return (e.clamp(0, 255) << 23).view(torch.float32)


def fp8_sim(x: torch.Tensor, block: int) -> torch.Tensor:
    """Block-wise FP8 e4m3 quant-dequant with power-of-two scales along the
    last dim: s = 2^ceil(log2(max(amax, 1e-4) / 448)), x -> bf16(e4m3(x/s) * s)."""
    shp = x.shape
    g = x.reshape(-1, shp[-1] // block, block)
    amax = g.abs().amax(-1, keepdim=True).clamp_min(1e-4)
    s = pow2_ceil(amax / 448.0)
    q = (g / s).clamp(-448.0, 448.0).to(torch.float8_e4m3fn).to(torch.float32)
    return bf16r(q * s).reshape(shp)


_E2M1 = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])


def _round_e2m1(a: torch.Tensor) -> torch.Tensor:
    """Round |values| <= 6 to the FP4 e2m1 grid, ties to the even mantissa."""
    grid = _E2M1.to(a.device)
    mag = a.abs()
    # Nearest grid point; on an exact midpoint take the even-mantissa entry
    # (grid indices 0, 2, 4, 6).
    d = (mag.unsqueeze(-1) - grid).abs()
    best = d.min(-1, keepdim=True).values
    cand = d == best
    idx = torch.arange(8, device=a.device)
    even = (idx % 2) == 0
    two = cand.sum(-1) > 1
    pick = torch.where(two.unsqueeze(-1), cand & even, cand)
    i = pick.to(torch.int64).argmax(-1)
    return torch.sign(a) * grid[i]


def fp4_sim(x: torch.Tensor, block: int) -> torch.Tensor:
    """Block-wise FP4 e2m1 quant-dequant with power-of-two scales:
    s = 2^ceil(log2(max(amax, 6 * 2^-126) / 6)), x -> bf16(e2m1(x/s) * s)."""
    shp = x.shape
    g = x.reshape(-1, shp[-1] // block, block)
    amax = g.abs().amax(-1, keepdim=True).clamp_min(6.0 * 2.0 ** -126)
    s = pow2_ceil(amax / 6.0)
    q = _round_e2m1((g / s).clamp(-6.0, 6.0))
    return bf16r(q * s).reshape(shp)


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    r = 1.0 / torch.sqrt((x * x).mean(-1, keepdim=True) + eps)
    return bf16r(x * r * w)


def rms_normalize(x: torch.Tensor, eps: float) -> torch.Tensor:
    r = 1.0 / torch.sqrt((x * x).mean(-1, keepdim=True) + eps)
    return bf16r(x * r)


_HAD: Dict[tuple, torch.Tensor] = {}


def hadamard(x: torch.Tensor, scale: float) -> torch.Tensor:
    """Walsh-Hadamard transform along the last dim (power of two), scaled,
    rounded to bf16."""
    n = x.shape[-1]
    key = (n, x.device)
    h = _HAD.get(key)
    if h is None:
        h = torch.ones(1, 1)
        while h.shape[0] < n:
            h = torch.cat([torch.cat([h, h], 1), torch.cat([h, -h], 1)], 0)
        h = h.to(x.device)
        _HAD[key] = h
    return bf16r((x @ h.t()) * scale)


def lin_bf16(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """x @ w^T in fp32, rounded to bf16 (bf16 weights, bf16 activations)."""
    return bf16r(x @ w.t())


def softplus(x: torch.Tensor) -> torch.Tensor:
    return torch.where(x > 20.0, x, torch.log1p(torch.exp(x)))


# ---------------------------------------------------------------------- rope

def rope_freqs(dim: int, seqlen: int, original_seq_len: int, base: float, factor: float,
               beta_fast: float, beta_slow: float, device) -> torch.Tensor:
    """cos / sin table [seqlen, dim/2, 2] (YaRN blending when
    original_seq_len > 0)."""
    half = dim // 2
    freqs = 1.0 / (torch.tensor(base, dtype=torch.float32) **
                   (torch.arange(0, dim, 2, dtype=torch.float32) / dim))
    if original_seq_len > 0:
        def corr(rot):
            return dim * math.log(original_seq_len / (rot * 2 * math.pi)) / (2 * math.log(base))

        lo = max(math.floor(corr(beta_fast)), 0.0)
        hi = min(math.ceil(corr(beta_slow)), dim - 1)
        if lo == hi:
            hi += 0.001
        ramp = ((torch.arange(half, dtype=torch.float32) - lo) / (hi - lo)).clamp(0, 1)
        smooth = 1 - ramp
        freqs = freqs / factor * (1 - smooth) + freqs * smooth
    ang = torch.arange(seqlen, dtype=torch.float32)[:, None] * freqs[None, :]
    return torch.stack([torch.cos(ang), torch.sin(ang)], -1).to(device)


def apply_rope(x: torch.Tensor, cs: torch.Tensor, rd: int, inverse: bool = False):
    """Rotate the last `rd` dims of x [..., n] as adjacent (even, odd) pairs;
    `cs` broadcasts as [..., rd/2, 2].  The rotated dims are rounded to
    bf16, the rest is left as is."""
    out = x.clone()
    a = x[..., -rd::2]
    b = x[..., -rd + 1::2]
    c, s = cs[..., 0], cs[..., 1]
    if inverse:
        s = -s
    out[..., -rd::2] = bf16r(a * c - b * s)
    out[..., -rd + 1::2] = bf16r(a * s + b * c)
    return out


# ----------------------------------------------------------- hyper-connections

def hc_coeffs(mixes: torch.Tensor, scale: torch.Tensor, base: torch.Tensor, hc: int,
              iters: int, eps: float):
    """mixes [T, (2+hc)*hc] -> pre [T, hc], post [T, hc], comb [T, hc, hc]."""
    pre = torch.sigmoid(mixes[:, :hc] * scale[0] + base[:hc]) + eps
    post = 2.0 * torch.sigmoid(mixes[:, hc:2 * hc] * scale[1] + base[hc:2 * hc])
    comb = (mixes[:, 2 * hc:] * scale[2] + base[2 * hc:]).view(-1, hc, hc)
    comb = torch.softmax(comb, dim=-1) + eps
    comb = comb / (comb.sum(-2, keepdim=True) + eps)
    for _ in range(max(0, iters - 1)):
        comb = comb / (comb.sum(-1, keepdim=True) + eps)
        comb = comb / (comb.sum(-2, keepdim=True) + eps)
    return pre, post, comb


# ------------------------------------------------------------------- weights

def _read_safetensors(path: str) -> Dict[str, torch.Tensor]:
    from safetensors.torch import load_file

    return {k: (v.float() if v.dtype != torch.int32 else v) for k, v in load_file(path).items()}


def _dequant_int4_bin(buf: bytes, off: int, rows: int, cols: int):
    """One matrix of an int4_bin expert file: packed nibbles [rows, cols/2]
    (low nibble = even column, value (q - 8) * scale) then bf16 scales
    [rows, cols/32]."""
    g = 32
    n_packed = rows * cols // 2
    n_scale = rows * (cols // g) * 2
    packed = np.frombuffer(buf, dtype=np.uint8, count=n_packed, offset=off)
    sc = np.frombuffer(buf, dtype=np.uint16, count=rows * (cols // g), offset=off + n_packed)
    scales = torch.from_numpy((sc.astype(np.uint32) << 16).view(np.float32).copy())
    lo = (packed & 0x0F).astype(np.int32) - 8
    hi = (packed >> 4).astype(np.int32) - 8
    q = np.stack([lo, hi], -1).reshape(rows, cols).astype(np.float32)
    w = torch.from_numpy(q).view(rows, cols // g, g) * scales.view(rows, cols // g, 1)
    return w.reshape(rows, cols), off + n_packed + n_scale


@dataclass
class DSV4Config:
    dim: int
    vocab: int
    n_layers: int
    n_heads: int
    head_dim: int
    rope_dim: int
    q_lora: int
    o_lora: int
    o_groups: int
    window: int
    compress_ratios: List[int]
    rope_theta: float
    compress_rope_theta: float
    rope_factor: float
    beta_fast: float
    beta_slow: float
    original_seq_len: int
    index_heads: int
    index_dim: int
    index_topk: int
    hc: int
    sinkhorn_iters: int
    hc_eps: float
    eps: float
    n_experts: int
    topk: int
    route_scale: float
    n_hash_layers: int
    swiglu_limit: float
    expert_inter: int
    eos_ids: List[int] = field(default_factory=list)

    @staticmethod
    def from_manifest(m: dict) -> "DSV4Config":
        assert m["arch"] == "deepseek_v4", m["arch"]
        return DSV4Config(
            dim=m["hidden_size"], vocab=m["vocab_size"], n_layers=m["num_layers"],
            n_heads=m["n_heads"], head_dim=m["head_dim"], rope_dim=m["rope_head_dim"],
            q_lora=m["q_lora_rank"], o_lora=m["o_lora_rank"], o_groups=m["o_groups"],
            window=m["window_size"], compress_ratios=list(m["compress_ratios"]),
            rope_theta=m["rope_theta"], compress_rope_theta=m["compress_rope_theta"],
            rope_factor=m["rope_factor"], beta_fast=m["beta_fast"], beta_slow=m["beta_slow"],
            original_seq_len=m["original_seq_len"], index_heads=m["index_n_heads"],
            index_dim=m["index_head_dim"], index_topk=m["index_topk"], hc=m["hc_mult"],
            sinkhorn_iters=m["hc_sinkhorn_iters"], hc_eps=m["hc_eps"], eps=m["rms_norm_eps"],
            n_experts=m["n_routed_experts"], topk=m["top_k"], route_scale=m["route_scale"],
            n_hash_layers=m["n_hash_layers"], swiglu_limit=m["swiglu_limit"],
            expert_inter=m["expert_intermediate"], eos_ids=list(m.get("eos_token_ids", [])))


# --------------------------------------------------------------- compressor

class Compressor:
    """Learned gated pooling of `ratio` tokens into one row (per-channel
    softmax over the candidate slots); ratio 4 overlaps with the previous
    block.  `rotate`: the indexer variant (Hadamard + FP4 instead of FP8)."""

    def __init__(self, w: Dict[str, torch.Tensor], prefix: str, d: int, rd: int, ratio: int,
                 rotate: bool, eps: float, device):
        self.wkv = w[prefix + "wkv.weight"].to(device)
        self.wgate = w[prefix + "wgate.weight"].to(device)
        self.ape = w[prefix + "ape"].to(device)
        self.norm = w[prefix + "norm.weight"].to(device)
        self.d, self.rd, self.ratio, self.rotate, self.eps = d, rd, ratio, rotate, eps
        self.overlap = ratio == 4
        self.coff = 2 if self.overlap else 1
        self.dev = device
        self.reset()

    def reset(self):
        cd = self.coff * self.d
        self.kv_state = torch.zeros(self.coff * self.ratio, cd, device=self.dev)
        self.sc_state = torch.full((self.coff * self.ratio, cd), float("-inf"), device=self.dev)

    def _finish(self, rows: torch.Tensor, pos0: torch.Tensor, freqs: torch.Tensor):
        rows = rmsnorm(bf16r(rows), self.norm, self.eps)
        rows = apply_rope(rows, freqs[pos0], self.rd)
        if self.rotate:
            return fp4_sim(hadamard(rows, self.d ** -0.5), 32)
        nr = self.d - self.rd
        out = rows.clone()
        out[:, :nr] = fp8_sim(rows[:, :nr], 64)
        return out

    @staticmethod
    def _pool(kv: torch.Tensor, sc: torch.Tensor) -> torch.Tensor:
        """kv, sc [B, slots, d] -> per-channel softmax-weighted sum [B, d]."""
        p = torch.softmax(sc, dim=1)
        return (p * kv).sum(1)

    def prefill(self, x: torch.Tensor, freqs: torch.Tensor) -> torch.Tensor:
        """x [s, dim] -> finished rows [s // ratio, d]; keeps the decode state."""
        s = x.shape[0]
        r, d, cd = self.ratio, self.d, self.coff * self.d
        kv = x @ self.wkv.t()
        sc = x @ self.wgate.t()
        rem = s % r
        cut = s - rem
        nblk = cut // r
        self.reset()
        if self.overlap and cut >= r:
            self.kv_state[:r] = kv[cut - r:cut]
            self.sc_state[:r] = sc[cut - r:cut] + self.ape
        off = r if self.overlap else 0
        if rem:
            self.kv_state[off:off + rem] = kv[cut:]
            self.sc_state[off:off + rem] = sc[cut:] + self.ape[:rem]
        if nblk == 0:
            return torch.zeros(0, d, device=x.device)
        kvb = kv[:cut].view(nblk, r, cd)
        scb = sc[:cut].view(nblk, r, cd) + self.ape
        if self.overlap:
            own_kv, own_sc = kvb[:, :, d:], scb[:, :, d:]
            prev_kv = torch.cat([torch.zeros(1, r, d, device=x.device), kvb[:-1, :, :d]], 0)
            prev_sc = torch.cat([torch.full((1, r, d), float("-inf"), device=x.device),
                                 scb[:-1, :, :d]], 0)
            rows = self._pool(torch.cat([prev_kv, own_kv], 1), torch.cat([prev_sc, own_sc], 1))
        else:
            rows = self._pool(kvb, scb)
        pos0 = torch.arange(nblk, device=x.device) * r
        return self._finish(rows, pos0, freqs)

    def decode(self, x: torch.Tensor, pos: int, freqs: torch.Tensor) -> Optional[torch.Tensor]:
        """One token (x [dim]) at position `pos`; a finished row when a block
        completes."""
        r, d, cd = self.ratio, self.d, self.coff * self.d
        kv = x @ self.wkv.t()
        sc = x @ self.wgate.t() + self.ape[pos % r]
        slot = (r + pos % r) if self.overlap else pos % r
        self.kv_state[slot] = kv
        self.sc_state[slot] = sc
        if (pos + 1) % r:
            return None
        if self.overlap:
            ckv = torch.cat([self.kv_state[:r, :d], self.kv_state[r:, d:]], 0)
            csc = torch.cat([self.sc_state[:r, :d], self.sc_state[r:, d:]], 0)
        else:
            ckv, csc = self.kv_state, self.sc_state
        row = self._pool(ckv[None], csc[None])
        if self.overlap:
            self.kv_state[:r] = self.kv_state[r:].clone()
            self.sc_state[:r] = self.sc_state[r:].clone()
        return self._finish(row, torch.tensor([pos + 1 - r], device=x.device), freqs)[0]


# ------------------------------------------------------------------ indexer

class Indexer:
    """Picks `topk` compressed rows per query: its own rotate-variant
    compressor over the same layer input, index heads (rope -> Hadamard ->
    FP4) scored against it with ReLU and learned per-head weights."""

    def __init__(self, w, cfg: DSV4Config, max_seq: int, device):
        self.h, self.d, self.rd = cfg.index_heads, cfg.index_dim, cfg.rope_dim
        self.topk, self.ratio = cfg.index_topk, 4
        self.wq_b = w["attn.indexer.wq_b.weight"].to(device)
        self.wproj = w["attn.indexer.weights_proj.weight"].to(device)
        self.comp = Compressor(w, "attn.indexer.compressor.", self.d, self.rd, 4, True, cfg.eps,
                               device)
        self.cache = torch.zeros(max_seq // 4, self.d, device=device)
        self.scale = self.d ** -0.5

    def reset(self):
        self.comp.reset()
        self.cache.zero_()

    def _q(self, qr: torch.Tensor, cs: torch.Tensor) -> torch.Tensor:
        """qr [T, q_lora], cs [T, rd/2, 2] -> [T, h, d]."""
        q = lin_bf16(qr, self.wq_b).view(-1, self.h, self.d)
        q = apply_rope(q, cs[:, None], self.rd)
        q = hadamard(q, self.d ** -0.5)
        return fp4_sim(q.reshape(q.shape[0], -1), 32).view(-1, self.h, self.d)

    def _w(self, x: torch.Tensor) -> torch.Tensor:
        return bf16r(lin_bf16(x, self.wproj) * (self.scale * self.h ** -0.5))

    def _scores(self, q: torch.Tensor, w: torch.Tensor, rows: int) -> torch.Tensor:
        """sum_h bf16(relu(bf16(q_h . kv_r)) * w_h), bf16 -> [T, rows]."""
        dots = bf16r(torch.einsum("thd,rd->thr", q, self.cache[:rows])).clamp_min(0.0)
        return bf16r(bf16r(dots * w[:, :, None]).sum(1))

    def prefill(self, x, qr, freqs, offset: int) -> torch.Tensor:
        """-> [s, min(topk, s // 4)] row indices (+offset), -1 where the row
        is not yet complete for that position."""
        s = x.shape[0]
        rows = self.comp.prefill(x, freqs)
        self.cache[:rows.shape[0]] = rows
        avail = s // 4
        k = min(self.topk, avail)
        if k == 0:
            return torch.zeros(s, 0, dtype=torch.long, device=x.device)
        q = self._q(qr, freqs[:s])
        sc = self._scores(q, self._w(x), avail)
        valid = ((torch.arange(s, device=x.device) + 1) // 4)[:, None]
        r = torch.arange(avail, device=x.device)[None, :]
        sc = torch.where(r >= valid, torch.full_like(sc, float("-inf")), sc)
        order = torch.sort(sc, dim=1, descending=True, stable=True).indices[:, :k]
        return torch.where(order >= valid, torch.full_like(order, -1), order + offset)

    def decode(self, x, qr, pos: int, freqs, offset: int) -> torch.Tensor:
        row = self.comp.decode(x, pos, freqs)
        if row is not None:
            self.cache[pos // 4] = row
        rows = (pos + 1) // 4
        k = min(self.topk, rows)
        if k == 0:
            return torch.zeros(0, dtype=torch.long, device=x.device)
        q = self._q(qr[None], freqs[pos:pos + 1])
        sc = self._scores(q, self._w(x[None]), rows)[0]
        return torch.sort(sc, descending=True, stable=True).indices[:k] + offset


# ---------------------------------------------------------------- attention

def sparse_attention(q: torch.Tensor, kv: torch.Tensor, idx: torch.Tensor, sink: torch.Tensor,
                     scale: float) -> torch.Tensor:
    """q [T, h, d]; kv [N, d]; idx [T, K] (-1 = masked); sink [h].
    Softmax over the gathered rows with the sink logit in the denominator
    only; output bf16 [T, h, d]."""
    valid = idx >= 0
    rows = kv[idx.clamp_min(0)]                       # [T, K, d]
    s = torch.einsum("thd,tkd->thk", q, rows) * scale
    s = s.masked_fill(~valid[:, None, :], float("-inf"))
    m = torch.maximum(s.amax(-1), sink[None, :])      # [T, h]
    e = torch.exp(s - m[..., None])
    denom = torch.exp(sink[None, :] - m) + e.sum(-1)
    p = e / denom[..., None]
    return bf16r(torch.einsum("thk,tkd->thd", p, rows))


class Attention:
    def __init__(self, w, cfg: DSV4Config, li: int, max_seq: int, device):
        self.cfg = cfg
        self.ratio = cfg.compress_ratios[li]
        self.h, self.hd, self.rd = cfg.n_heads, cfg.head_dim, cfg.rope_dim
        self.win = cfg.window
        g = lambda n: w[n].to(device)  # noqa: E731
        self.wq_a, self.q_norm = g("attn.wq_a.weight"), g("attn.q_norm.weight")
        self.wq_b, self.wkv = g("attn.wq_b.weight"), g("attn.wkv.weight")
        self.kv_norm, self.sink = g("attn.kv_norm.weight"), g("attn.attn_sink")
        self.wo_a, self.wo_b = g("attn.wo_a.weight"), g("attn.wo_b.weight")
        self.comp = (Compressor(w, "attn.compressor.", self.hd, self.rd, self.ratio, False,
                                cfg.eps, device) if self.ratio > 0 else None)
        self.idx = Indexer(w, cfg, max_seq, device) if self.ratio == 4 else None
        theta = cfg.compress_rope_theta if self.ratio > 0 else cfg.rope_theta
        orig = cfg.original_seq_len if self.ratio > 0 else 0
        self.freqs = rope_freqs(self.rd, max_seq, orig, theta, cfg.rope_factor, cfg.beta_fast,
                                cfg.beta_slow, device)
        self.scale = self.hd ** -0.5
        n_comp = max_seq // self.ratio if self.ratio > 0 else 0
        self.cache = torch.zeros(self.win + n_comp, self.hd, device=device)
        self.dev = device

    def reset(self):
        self.cache.zero_()
        if self.comp is not None:
            self.comp.reset()
        if self.idx is not None:
            self.idx.reset()

    def _qr(self, x):
        return rmsnorm(lin_bf16(x, self.wq_a), self.q_norm, self.cfg.eps)

    def _q(self, qr, cs):
        q = rms_normalize(lin_bf16(qr, self.wq_b).view(-1, self.h, self.hd), self.cfg.eps)
        return apply_rope(q, cs[:, None], self.rd)

    def _kv(self, x, cs):
        kv = apply_rope(rmsnorm(lin_bf16(x, self.wkv), self.kv_norm, self.cfg.eps), cs, self.rd)
        nr = self.hd - self.rd
        out = kv.clone()
        out[:, :nr] = fp8_sim(kv[:, :nr], 64)
        return out

    def _out(self, o, cs):
        """inverse rope + grouped low-rank O: o [T, h, hd] -> [T, dim]."""
        o = apply_rope(o, cs[:, None], self.rd, inverse=True)
        G = self.cfg.o_groups
        og = o.reshape(o.shape[0], G, -1)
        wa = self.wo_a.view(G, self.cfg.o_lora, -1)
        mid = bf16r(torch.einsum("tgd,gjd->tgj", og, wa)).reshape(o.shape[0], -1)
        return lin_bf16(mid, self.wo_b)

    def prefill(self, x: torch.Tensor) -> torch.Tensor:
        s = x.shape[0]
        dev = x.device
        cs = self.freqs[:s]
        qr = self._qr(x)
        kv = self._kv(x, cs)
        t = torch.arange(s, device=dev)
        win_idx = t[:, None] - (self.win - 1) + torch.arange(self.win, device=dev)[None, :]
        # Window slots in increasing position, padded with -1 at the end.
        n_valid = torch.clamp(t + 1, max=self.win)[:, None]
        lo = torch.clamp(t - (self.win - 1), min=0)[:, None]
        win_idx = lo + torch.arange(self.win, device=dev)[None, :]
        win_idx = torch.where(torch.arange(self.win, device=dev)[None, :] < n_valid, win_idx,
                              torch.full_like(win_idx, -1))
        kv_all = kv
        idx = win_idx
        comp_rows = None
        if self.ratio > 0:
            if self.idx is not None:
                cidx = self.idx.prefill(x, qr, self.freqs, s)
            else:
                n = s // self.ratio
                r = torch.arange(n, device=dev)[None, :]
                valid = ((t + 1) // self.ratio)[:, None]
                cidx = torch.where(r < valid, r + s, torch.full_like(r.expand(s, n), -1))
            comp_rows = self.comp.prefill(x, self.freqs)
            kv_all = torch.cat([kv, comp_rows], 0)
            idx = torch.cat([win_idx, cidx], 1)
        o = sparse_attention(self._q(qr, cs), kv_all, idx, self.sink, self.scale)
        out = self._out(o, cs)
        # Decode state: the raw-latent ring and the compressed rows.
        for p in range(max(0, s - self.win), s):
            self.cache[p % self.win] = kv[p]
        if comp_rows is not None and comp_rows.shape[0]:
            self.cache[self.win:self.win + comp_rows.shape[0]] = comp_rows
        return out

    def decode(self, x: torch.Tensor, pos: int) -> torch.Tensor:
        """x [dim] at absolute position `pos` -> [dim]."""
        dev = x.device
        cs = self.freqs[pos:pos + 1]
        qr = self._qr(x[None])
        self.cache[pos % self.win] = self._kv(x[None], cs)[0]
        if pos >= self.win - 1:
            idx = torch.arange(self.win, device=dev)
        else:
            idx = torch.cat([torch.arange(pos + 1, device=dev),
                             torch.full((self.win - pos - 1,), -1, device=dev)])
        if self.ratio > 0:
            if self.idx is not None:
                cidx = self.idx.decode(x, qr[0], pos, self.freqs, self.win)
            else:
                cidx = torch.arange((pos + 1) // self.ratio, device=dev) + self.win
            row = self.comp.decode(x, pos, self.freqs)
            if row is not None:
                self.cache[self.win + pos // self.ratio] = row
            idx = torch.cat([idx, cidx])
        o = sparse_attention(self._q(qr, cs), self.cache, idx[None], self.sink, self.scale)
        return self._out(o, cs)[0]


# -------------------------------------------------------------------- MoE

class MoE:
    def __init__(self, w, cfg: DSV4Config, li: int, expert_dir: str, device):
        self.cfg = cfg
        self.gate = w["ffn.gate.weight"].to(device)
        self.hash = li < cfg.n_hash_layers
        self.bias = None if self.hash else w["ffn.gate.bias"].to(device)
        self.tid2eid = w["ffn.gate.tid2eid"].to(device).long() if self.hash else None
        d, f = cfg.dim, cfg.expert_inter
        w1, w3, w2 = [], [], []
        for e in [f"expert_{i:03d}.bin" for i in range(cfg.n_experts)] + ["expert_shared.bin"]:
            buf = open(os.path.join(expert_dir, e), "rb").read()
            a, off = _dequant_int4_bin(buf, 0, f, d)
            b, off = _dequant_int4_bin(buf, off, f, d)
            c, off = _dequant_int4_bin(buf, off, d, f)
            w1.append(a)
            w3.append(b)
            w2.append(c)
        self.w1 = torch.stack(w1).to(device)  # [E+1, f, d]; the last is shared
        self.w3 = torch.stack(w3).to(device)
        self.w2 = torch.stack(w2).to(device)

    def _expert(self, x, e, route_w):
        """x [T, d]; e [T] expert ids; route_w [T] or None -> bf16 [T, d]."""
        g = bf16r(torch.einsum("td,tfd->tf", x, self.w1[e]))
        u = bf16r(torch.einsum("td,tfd->tf", x, self.w3[e]))
        lim = self.cfg.swiglu_limit
        if lim > 0:
            u = u.clamp(-lim, lim)
            g = g.clamp_max(lim)
        h = g / (1 + torch.exp(-g)) * u
        if route_w is not None:
            h = h * route_w[:, None]
        return bf16r(torch.einsum("tf,tdf->td", bf16r(h), self.w2[e]))

    def __call__(self, x: torch.Tensor, ids: Optional[torch.Tensor]) -> torch.Tensor:
        cfg = self.cfg
        scores = torch.sqrt(softplus(x @ self.gate.t()))
        if self.hash:
            sel = self.tid2eid[ids]
        else:
            sel = torch.sort(scores + self.bias, dim=-1, descending=True, stable=True
                             ).indices[:, :cfg.topk]
        wts = scores.gather(1, sel)
        wts = wts / wts.sum(-1, keepdim=True) * cfg.route_scale
        y = torch.zeros_like(x)
        k = sel.shape[1]
        for j in range(k):
            # A later duplicate of the same expert replaces this contribution.
            dup = torch.zeros(sel.shape[0], dtype=torch.bool, device=x.device)
            for j2 in range(j + 1, k):
                dup |= sel[:, j2] == sel[:, j]
            out = self._expert(x, sel[:, j], wts[:, j])
            y = y + torch.where(dup[:, None], torch.zeros_like(out), out)
        shared = torch.full((x.shape[0],), cfg.n_experts, dtype=torch.long, device=x.device)
        y = y + self._expert(x, shared, None)
        return bf16r(y)


# -------------------------------------------------------------------- model

class DSV4Model:
    """Single-sequence DeepSeek-V4 over an export directory (manifest.json,
    embed / head safetensors, per-layer shells, int4_bin experts)."""

    def __init__(self, path: str, device="cpu", max_seq: int = 256):
        self.path = path
        with open(os.path.join(path, "manifest.json")) as f:
            self.cfg = cfg = DSV4Config.from_manifest(json.load(f))
        dev = torch.device(device)
        self.dev = dev
        self.embed = _read_safetensors(os.path.join(path, "embed.safetensors"))[
            "embed.weight"].to(dev)
        hd = _read_safetensors(os.path.join(path, "head.safetensors"))
        self.head_w, self.norm_w = hd["head.weight"].to(dev), hd["norm.weight"].to(dev)
        self.hc_head_fn, self.hc_head_base = hd["hc_head_fn"].to(dev), hd["hc_head_base"].to(dev)
        self.hc_head_scale = hd["hc_head_scale"].to(dev)
        self.layers = []
        for li in range(cfg.n_layers):
            w = _read_safetensors(os.path.join(path, "shells", f"layer_{li:02d}.safetensors"))
            self.layers.append({
                "attn": Attention(w, cfg, li, max_seq, dev),
                "attn_norm": w["attn_norm.weight"].to(dev),
                "ffn_norm": w["ffn_norm.weight"].to(dev),
                "moe": MoE(w, cfg, li, os.path.join(path, "experts", f"layer_{li:02d}"), dev),
                "hc_attn": (w["hc_attn_fn"].to(dev), w["hc_attn_base"].to(dev),
                            w["hc_attn_scale"].to(dev)),
                "hc_ffn": (w["hc_ffn_fn"].to(dev), w["hc_ffn_base"].to(dev),
                           w["hc_ffn_scale"].to(dev)),
            })
        self.max_seq = max_seq

    def reset(self):
        for L in self.layers:
            L["attn"].reset()

    # -------------------------------------------------------- HC wiring
    def _hc_pre(self, copies: torch.Tensor, params):
        """copies [T, hc, dim] -> (reduced input [T, dim], post, comb)."""
        fn, base, scale = params
        cfg = self.cfg
        if copies.is_cuda:
            from .. import ops

            y, post, comb, _ = ops.hc_pre(copies, fn, base, scale, cfg.sinkhorn_iters,
                                          cfg.hc_eps, cfg.eps)
            return y, post, comb
        flat = copies.reshape(copies.shape[0], -1)
        r = 1.0 / torch.sqrt((flat * flat).mean(-1, keepdim=True) + cfg.eps)
        mixes = (flat @ fn.t()) * r
        pre, post, comb = hc_coeffs(mixes, scale, base, cfg.hc, cfg.sinkhorn_iters, cfg.hc_eps)
        y = bf16r((pre[:, :, None] * copies).sum(1))
        return y, post, comb

    @staticmethod
    def _hc_post(sub, copies, post, comb):
        """new[j] = bf16(post[j] * sub + sum_i comb[i][j] * old[i])."""
        return bf16r(post[:, :, None] * sub[:, None, :] +
                     torch.einsum("tij,tid->tjd", comb, copies))

    def _layer(self, li: int, copies, ids, pos: Optional[int]):
        L = self.layers[li]
        cfg = self.cfg
        y, post, comb = self._hc_pre(copies, L["hc_attn"])
        y = rmsnorm(y, L["attn_norm"], cfg.eps)
        a = L["attn"].prefill(y) if pos is None else L["attn"].decode(y[0], pos)[None]
        copies = self._hc_post(a, copies, post, comb)
        y, post, comb = self._hc_pre(copies, L["hc_ffn"])
        y = rmsnorm(y, L["ffn_norm"], cfg.eps)
        return self._hc_post(L["moe"](y, ids), copies, post, comb)

    def _logits(self, copies: torch.Tensor) -> torch.Tensor:
        """Head over the copies of each row [T, hc, dim] -> fp32 [T, vocab]."""
        cfg = self.cfg
        flat = copies.reshape(copies.shape[0], -1)
        r = 1.0 / torch.sqrt((flat * flat).mean(-1, keepdim=True) + cfg.eps)
        mixes = flat @ self.hc_head_fn.t()
        pre = torch.sigmoid(mixes * r * self.hc_head_scale[0] + self.hc_head_base) + cfg.hc_eps
        y = bf16r((pre[:, :, None] * copies).sum(1))
        return rmsnorm(y, self.norm_w, cfg.eps) @ self.head_w.t()

    # ----------------------------------------------------------- public
    def prefill(self, ids: Sequence[int]) -> torch.Tensor:
        """Logits of the last prompt position (fp32 [vocab]); fills the
        decode state."""
        self.reset()
        t = torch.tensor(list(ids), dtype=torch.long, device=self.dev)
        copies = self.embed[t][:, None, :].expand(-1, self.cfg.hc, -1).contiguous()
        for li in range(len(self.layers)):
            copies = self._layer(li, copies, t, None)
        return self._logits(copies[-1:])[0]

    def decode(self, token: int, pos: int) -> torch.Tensor:
        t = torch.tensor([token], dtype=torch.long, device=self.dev)
        copies = self.embed[t][:, None, :].expand(-1, self.cfg.hc, -1).contiguous()
        for li in range(len(self.layers)):
            copies = self._layer(li, copies, t, pos)
        return self._logits(copies)[0]

    def generate(self, prompt: Sequence[int], max_new_tokens: int) -> List[int]:
        """Greedy tokens after the prompt (stops at an EOS id)."""
        logits = self.prefill(prompt)
        out = [int(torch.argmax(logits))]
        while len(out) < max_new_tokens and out[-1] not in self.cfg.eos_ids:
            logits = self.decode(out[-1], len(prompt) + len(out) - 1)
            out.append(int(torch.argmax(logits)))
        return out
