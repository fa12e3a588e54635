"""Activation-sparse SwiGLU FFN for single-token decode (optional, off by
default; dense is the correctness baseline).

Gate first; lane i of the intermediate is active when
``|silu(g_i)| >= tau_i * max_j |silu(g_j)|`` with one global tau (CATS) or
per-channel taus calibrated offline (CHESS); up is computed only for active
lanes and the down projection runs as an AXPY over a transposed,
re-quantised down weight, so an inactive lane's weights are never read.
Reference: crates/cascadia-int4-gemm/src/ffn_sparsity.rs:106-186 (mask),
:253 (rows-subset GEMV), ffn_axpy.rs:167-273 (AXPY down), :342
(transpose + re-quantise), bin calibrate_ffn_thresholds (CHESS taus).
The GPU path is ``csrc/ffn_sparse.cu``.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from ..quant import Int4Weight


def transpose_requantize(down: Int4Weight, group_size: Optional[int] = None) -> Int4Weight:
    """down [H, I] (groups along I) -> down^T [I, H] with groups along H.
    Each weight is rounded a second time into its new group's scale."""
    gs = group_size or down.group_size
    return Int4Weight.quantize(down.dequant_bf16().float().t().contiguous(), gs)


def build_active_mask(gate: torch.Tensor, tau) -> Tuple[torch.Tensor, torch.Tensor]:
    """(silu(gate) [I], ascending active lane indices) for one token."""
    s = torch.nn.functional.silu(gate.float())
    mx = s.abs().max()
    t = tau if isinstance(tau, torch.Tensor) else torch.full_like(s, float(tau))
    on = (t <= 0) | (s.abs() >= t.float() * mx)
    return s, torch.nonzero(on).flatten()


def calibrate_tau(gate_samples: torch.Tensor, active_frac: float) -> torch.Tensor:
    """Per-channel taus (CHESS) from gate outputs [N tokens, I]: tau_i is the
    (1 - active_frac) quantile of |silu(g_i)| / max_j |silu(g_j)| over the
    tokens, so lane i is active on about ``active_frac`` of them."""
    s = torch.nn.functional.silu(gate_samples.float()).abs()
    rel = s / s.max(dim=1, keepdim=True).values.clamp_min(1e-30)
    return torch.quantile(rel, 1.0 - active_frac, dim=0)


class SparseFFN:
    """Prepared weights of one SwiGLU FFN for the sparse single-token path."""

    def __init__(self, gate: Int4Weight, up: Int4Weight, down: Int4Weight, device,
                 tau_all: float = 0.05, tau: Optional[torch.Tensor] = None,
                 down_group: int = 32):
        assert gate.group_size == up.group_size
        self.I, self.H = gate.n, gate.k
        self.gs = gate.group_size
        self.device = torch.device(device)
        self.tau_all = float(tau_all)
        self.tau = tau.float().to(self.device) if tau is not None else None
        # The transposed down is re-quantised in groups of 32 along H (its
        # second rounding; finer groups keep that error small).
        self.down_gs = down_group
        down_t = transpose_requantize(down, down_group)
        self.down_t_w = down_t
        if self.device.type == "cuda":
            def prep(w):
                return (w.packed.to(self.device).contiguous(),
                        w.scales.to(torch.bfloat16).to(self.device).contiguous())
            self.gate, self.up, self.down_t = prep(gate), prep(up), prep(down_t)
            self.iwork = torch.zeros(2 * self.I + 1, dtype=torch.int32, device=self.device)
            self.fwork = torch.zeros(3 * self.I + self.H, dtype=torch.float32, device=self.device)
        else:
            self.gate_ref = gate.dequant_bf16().float()
            self.up_ref = up.dequant_bf16().float()
            self.down_t_ref = down_t.dequant_bf16().float()

    def __call__(self, x: torch.Tensor, residual: Optional[torch.Tensor] = None,
                 out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """x [1, H] bf16 -> [1, H] bf16 = FFN(x) (+ residual)."""
        assert x.shape[0] == 1, "the sparse FFN path serves one token"
        if out is None:
            out = torch.empty_like(x)
        if self.device.type == "cuda":
            from . import LAUNCHES, ext

            ext().ffn_sparse_forward(x.contiguous(), self.gate[0], self.gate[1], self.up[0],
                                     self.up[1], self.down_t[0], self.down_t[1], self.tau,
                                     self.tau_all, residual, out, self.iwork, self.fwork, self.gs,
                                     self.down_gs)
            LAUNCHES.add(5)
            return out
        xf = x[0].float()
        g = self.gate_ref @ xf
        s, act = build_active_mask(g, self.tau if self.tau is not None else self.tau_all)
        a = s[act] * (self.up_ref[act] @ xf)
        y = a @ self.down_t_ref[act]
        if residual is not None:
            y = y + residual[0].float()
        out.copy_(y.to(torch.bfloat16).view(1, -1))
        return out

    def active_fraction(self, x: torch.Tensor) -> float:
        """Fraction of lanes active for token x (CPU-prepared FFNs)."""
        g = self.gate_ref @ x[0].float()
        _, act = build_active_mask(g, self.tau if self.tau is not None else self.tau_all)
        return act.numel() / self.I
