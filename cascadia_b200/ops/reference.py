"""Plain-PyTorch fp32 restatement of every device op.

These are the CPU oracle for the kernel tests and the compute path of the CPU
engine (the BASELINE CPU config: Llama-3.2-1B shape, 2-stage loopback
pipeline).  They follow the reference's math:

* INT4 dequant ``(q - 8) * scale``: crates/cascadia-int4-gemm/src/kernel.rs:46-70
* RMSNorm: crates/cascadia-int4-gemm/src/shell.rs:371-394
* RoPE / llama3 scaling: crates/cascadia-engine-openvino/src/rotary.rs:111-185
* sampling: crates/cascadia-engine-sparse-moe/src/sampling.rs:52-187
"""
from __future__ import annotations

import math
from typing import List, Optional, Sequence

import torch

from ..quant import Int4Weight


def dequant(w: Int4Weight) -> torch.Tensor:
    """bf16-rounded dequantised weight [N, K] (what the GPU kernel feeds the MMA)."""
    return w.dequant_bf16()


def linear(x: torch.Tensor, w: Int4Weight) -> torch.Tensor:
    """x[M, K] @ dequant(W)^T in fp32; returns fp32."""
    return x.float() @ w.dequant_bf16().float().t()


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    inv = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return xf * inv * w.float()


def silu_mul(g: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
    g = g.float()
    return g / (1.0 + torch.exp(-g)) * u.float()


def apply_rope(x: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor, rot: int,
               interleaved: bool = False) -> torch.Tensor:
    """x: [T, H, D] float; rotate the first `rot` dims of each head."""
    half = rot // 2
    cs = cos_sin[positions.long()]  # [T, rot]
    cos = cs[:, :half].unsqueeze(1)
    sin = cs[:, half:].unsqueeze(1)
    out = x.clone()
    if interleaved:
        x0 = x[..., 0:rot:2]
        x1 = x[..., 1:rot:2]
        out[..., 0:rot:2] = x0 * cos - x1 * sin
        out[..., 1:rot:2] = x1 * cos + x0 * sin
    else:
        x0 = x[..., :half]
        x1 = x[..., half:rot]
        out[..., :half] = x0 * cos - x1 * sin
        out[..., half:rot] = x1 * cos + x0 * sin
    return out


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q_pos: torch.Tensor,
              scale: float, window: int = 0, sinks: int = 0) -> torch.Tensor:
    """Causal GQA attention for one sequence.

    q: [Tq, Hq, D], k/v: [Tk, Hkv, D] (positions 0..Tk-1), q_pos: [Tq].
    window > 0: a query at q sees keys q - window < k <= q and k < sinks.
    """
    tq, hq, d = q.shape
    tk, hkv, _ = k.shape
    g = hq // hkv
    kf = k.float().repeat_interleave(g, dim=1)  # [Tk, Hq, D]
    vf = v.float().repeat_interleave(g, dim=1)
    s = torch.einsum("qhd,khd->hqk", q.float(), kf) * scale
    kpos = torch.arange(tk)
    mask = kpos[None, :] > q_pos.long()[:, None]  # [Tq, Tk]
    if window > 0:
        far = kpos[None, :] <= q_pos.long()[:, None] - window
        mask = mask | (far & (kpos[None, :] >= sinks))
    s = s.masked_fill(mask[None], float("-inf"))
    p = torch.softmax(s, dim=-1)
    return torch.einsum("hqk,khd->qhd", p, vf)


def argmax(logits: torch.Tensor) -> torch.Tensor:
    """Row argmax, lowest index on ties (the reference's strict `>` scan)."""
    return torch.argmax(logits.float(), dim=-1).to(torch.int32)


# ----------------------------------------------------------------- sampling

_MASK64 = (1 << 64) - 1


def xorshift64_next(state: List[int]) -> int:
    """xorshift64* step (crates/cascadia-engine-sparse-moe/src/sampling.rs:191)."""
    x = state[0]
    x ^= (x << 13) & _MASK64
    x ^= x >> 7
    x ^= (x << 17) & _MASK64
    state[0] = x
    return (x * 0x2545F4914F6CDD1D) & _MASK64


def next_uniform(state: List[int]) -> float:
    r = xorshift64_next(state)
    return float(r >> 40) / float(1 << 24)


def init_rng(seed: Optional[int]) -> List[int]:
    if seed is not None:
        return [max(int(seed) & _MASK64, 1)]
    import time

    t = time.time_ns()
    return [max(((t % 10**9) | ((t // 10**9) << 32)) & _MASK64, 1)]


def apply_penalties(work: torch.Tensor, history: Sequence[int], rep_pen: float, rep_window: int,
                    freq_pen: float, pres_pen: float) -> torch.Tensor:
    work = work.clone()
    if abs(rep_pen - 1.0) > 1.1920929e-07:
        start = 0 if rep_window == 0 else max(0, len(history) - rep_window)
        for tok in history[start:]:
            if 0 <= tok < work.numel():
                l = float(work[tok])
                work[tok] = l / rep_pen if l > 0 else l * rep_pen
    if freq_pen != 0.0 or pres_pen != 0.0:
        seen = set()
        for tok in history:
            if 0 <= tok < work.numel():
                work[tok] -= freq_pen
                if tok not in seen:
                    seen.add(tok)
                    work[tok] -= pres_pen
    return work


def sample(logits: torch.Tensor, history: Sequence[int], temperature: float, top_p: float,
           top_k: int, freq_pen: float, pres_pen: float, rep_pen: float, rep_window: int,
           rng_state: List[int]) -> int:
    """Sample one token with the reference's exact semantics and PRNG."""
    work = apply_penalties(logits.float().flatten(), history, rep_pen, rep_window, freq_pen,
                           pres_pen)
    if temperature <= 0.0:
        return int(torch.argmax(work))
    work = work / temperature
    work = torch.softmax(work, dim=0)
    n = work.numel()
    if 0 < top_k < n:
        idx = torch.argsort(work, descending=True, stable=True)
        keep = torch.zeros(n, dtype=torch.bool)
        keep[idx[:top_k]] = True
        work = torch.where(keep, work, torch.zeros_like(work))
        s = work.sum()
        if s > 0:
            work = work / s
    if 0.0 < top_p < 1.0:
        idx = torch.argsort(work, descending=True, stable=True)
        cum = torch.cumsum(work[idx], 0)
        cut = int(torch.searchsorted(cum, torch.tensor(top_p, dtype=cum.dtype)).item())
        keep = torch.zeros(n, dtype=torch.bool)
        keep[idx[: min(n, cut + 1)]] = True
        work = torch.where(keep, work, torch.zeros_like(work))
        s = work.sum()
        if s > 0:
            work = work / s
    u = next_uniform(rng_state)
    cum = torch.cumsum(work, 0)
    hit = torch.nonzero(cum >= u)
    return int(hit[0]) if hit.numel() else n - 1


def spec_verify(target: Sequence[int], draft: Sequence[int]):
    """Greedy acceptance: longest matching prefix plus the correction token."""
    acc = 0
    while acc < len(draft) and draft[acc] == target[acc]:
        acc += 1
    return list(draft[:acc]) + [int(target[acc])]
