"""Device ops: thin wrappers over the sm_100a kernels in ``cascadia_b200._C``.

Every function takes CUDA tensors and launches one of our own kernels on the
current stream.  There is no silent fallback: if the extension is missing on a
machine with a GPU, ``ext()`` raises.  The CPU reference implementations of
the same math (used by the CPU engine and as test oracles) live in
:mod:`cascadia_b200.ops.reference` and are only used for CPU tensors.
"""
from __future__ import annotations

import math
import os
import threading
from typing import Optional

import torch

from . import debug as _dbg

_EXT = None
_EXT_ERR: Optional[BaseException] = None
_LOCK = threading.Lock()


def ext():
    """Return the compiled extension module or raise a clear error."""
    global _EXT, _EXT_ERR
    if _EXT is not None:
        return _EXT
    with _LOCK:
        if _EXT is None:
            try:
                from cascadia_b200 import _C  # type: ignore

                _EXT = _C
            except BaseException as e:  # pragma: no cover - depends on build
                _EXT_ERR = e
                raise RuntimeError(
                    "cascadia_b200 CUDA extension is not built; run "
                    "`python setup.py build_ext --inplace` (sm_100a)") from e
    return _EXT


def ext_available() -> bool:
    try:
        ext()
        return True
    except RuntimeError:
        return False


# ----------------------------------------------------------------- launch count
class LaunchCounter:
    """Counts our own kernel launches issued through this module (e.g. while a
    CUDA graph is captured, to know how many kernels one replay runs)."""

    def __init__(self):
        self.count = 0
        self.active = False

    def reset(self):
        self.count = 0
        self.active = False

    def start(self):
        self.count = 0
        self.active = True

    def stop(self) -> int:
        self.active = False
        return self.count

    def add(self, n: int = 1):
        if self.active:
            self.count += n


LAUNCHES = LaunchCounter()


# ----------------------------------------------------------------- status word
_STATUS: dict = {}


def status_buffer(device: torch.device) -> torch.Tensor:
    """Per-device int32 status word written by bounded device-side waits."""
    key = torch.device(device).index or 0
    buf = _STATUS.get(key)
    if buf is None:
        buf = torch.zeros(1, dtype=torch.int32, device=device)
        _STATUS[key] = buf
    return buf


# Codes written by the kernels' bounded waits (csrc/common.cuh StatusCode).
STATUS_NAMES = {
    101: "GEMM weight/activation load timed out",
    102: "GEMM MMA issue timed out",
    103: "GEMM epilogue timed out",
    104: "GEMM dequantisation timed out",
    201: "attention load timed out",
    301: "peer (NVLink) signal timed out",
    401: "MoE expert-parallel exchange timed out",
}


def status_name(code: int) -> str:
    return STATUS_NAMES.get(int(code), "unknown device status")


def read_status(device: torch.device, clear: bool = True) -> int:
    buf = status_buffer(device)
    v = int(buf.item())
    if clear and v != 0:
        buf.zero_()
    return v


# ----------------------------------------------------------------- GEMM
EPI_STORE, EPI_SILU, EPI_RESID = 0, 1, 2


class GemmWorkspace:
    """Split-K scratch (fp32 partials + per-tile counters) for one stream.

    The counters return to zero at the end of every GEMM, so a workspace can
    be reused by any number of back-to-back launches on the same stream (and
    inside CUDA graphs).  Concurrent streams need their own workspace.
    """

    def __init__(self, device, max_floats: int = 1 << 24, max_counters: int = 1 << 16):
        self.device = torch.device(device)
        self.ws = torch.empty(max(1, max_floats), dtype=torch.float32, device=self.device)
        self.counters = torch.zeros(max_counters, dtype=torch.int32, device=self.device)
        # Buffers replaced by a larger one stay alive: a captured CUDA graph
        # may still point at them.
        self._retired = []

    def ensure(self, floats: int, counters: int):
        if floats > self.ws.numel():
            self._retired.append(self.ws)
            self.ws = torch.empty(floats, dtype=torch.float32, device=self.device)
        if counters > self.counters.numel():
            self._retired.append(self.counters)
            self.counters = torch.zeros(counters, dtype=torch.int32, device=self.device)


_WS: dict = {}


def default_workspace(device) -> GemmWorkspace:
    key = (torch.device(device).index or 0, torch.cuda.current_stream(device).cuda_stream)
    ws = _WS.get(key)
    if ws is None:
        ws = GemmWorkspace(device)
        _WS[key] = ws
    return ws


def w4a16_gemm(x: torch.Tensor, blob: torch.Tensor, n: int, group_size: int = 128,
               epilogue: int = EPI_STORE, residual: Optional[torch.Tensor] = None,
               out: Optional[torch.Tensor] = None, workspace: Optional[GemmWorkspace] = None,
               splits: int = 0) -> torch.Tensor:
    """Y = X @ dequant(W)^T with a fused epilogue.  Up to 8 rows run the
    small-M kernel (register-fed warp MMAs), larger M the tcgen05 kernel;
    ``splits > 0`` forces the tcgen05 kernel with that split-K factor."""
    m, k = x.shape
    e = ext()
    n_out = n // 2 if epilogue == EPI_SILU else n
    if out is None:
        out = torch.empty(m, n_out, dtype=torch.bfloat16, device=x.device)
    ws = workspace or default_workspace(x.device)
    ws.ensure(e.w4a16_workspace_floats(m, n, k, splits), e.w4a16_counter_count(m, n))
    e.w4a16_gemm(x, blob, out, n, group_size, epilogue, residual, ws.ws, ws.counters,
                 status_buffer(x.device), splits)
    LAUNCHES.add(1)
    return out


def bf16_gemm(x: torch.Tensor, w: torch.Tensor, residual: Optional[torch.Tensor] = None,
              out: Optional[torch.Tensor] = None, workspace: Optional[GemmWorkspace] = None,
              splits: int = 0) -> torch.Tensor:
    """Y = X @ W^T (+ residual) on the tcgen05 bf16 GEMM (both operands
    TMA-staged in shared memory, fp32 accumulator in tensor memory, split-K
    with a deterministic last-CTA reduction for small tile counts)."""
    m, k = x.shape
    n = w.shape[0]
    if x.stride(1) != 1 or (x.stride(0) * 2) % 16 or x.data_ptr() % 16:
        x = x.contiguous()
    if out is None:
        out = torch.empty(m, n, dtype=torch.bfloat16, device=x.device)
    e = ext()
    plan = e.bf16_gemm_plan(m, n, k, splits)
    ws = workspace or default_workspace(x.device)
    ws.ensure(plan[4], plan[5])
    e.bf16_gemm(x, w, out, residual, ws.ws, ws.counters, status_buffer(x.device), splits)
    LAUNCHES.add(1)
    return out


def hc_pre(copies: torch.Tensor, fn: torch.Tensor, base: torch.Tensor, scale: torch.Tensor,
           iters: int, hc_eps: float, norm_eps: float):
    """DeepSeek-V4 Hyper-Connections pre-mix in one kernel: copies
    [T, hc, dim] fp32 -> (y [T, dim] bf16-valued, post [T, hc],
    comb [T, hc, hc], pre [T, hc])."""
    out = ext().hc_pre(copies.contiguous(), fn, base, scale, iters, hc_eps, norm_eps)
    LAUNCHES.add(1)
    return out


def _gemv_max_m() -> int:
    try:
        return int(os.environ.get("CASCADIA_GEMV_MAX_M", "8"))
    except ValueError:
        return 8


FUSE_ROPE = os.environ.get("CASCADIA_FUSE_ROPE", "1") != "0"


def rope_fusable(m: int, head_dim: int, rot: int, group_size: int) -> bool:
    """The q/k/v GEMM can carry RoPE and the KV write in its epilogue: the
    tcgen05 kernel runs (more rows than the small-M kernel takes), head_dim
    128 with full rotate-half rotation."""
    return (FUSE_ROPE and m > _gemv_max_m() and head_dim == 128 and rot == 128
            and group_size in (32, 128))


def w4a16_gemm_rope_kv(x, blob, n, group_size, out, positions, cos_sin, slots, k_cache,
                       v_cache, layer, hq, hkv, workspace: Optional[GemmWorkspace] = None):
    """The q/k/v projection with RoPE + paged-KV write in its epilogue: out
    gets the rotated q heads; K and V go straight into the caches."""
    m, k = x.shape
    if _dbg.ENABLED and not torch.cuda.is_current_stream_capturing():
        _dbg.check_range("kv slots", slots[:m], 0, k_cache.shape[1] * 16, allow=(-1,))
        _dbg.check_range("positions", positions[:m], 0, cos_sin.shape[0])
        _dbg.check_range("layer", torch.tensor([layer]), 0, k_cache.shape[0])
    e = ext()
    ws = workspace or default_workspace(x.device)
    ws.ensure(e.w4a16_workspace_floats(m, n, k, 0), e.w4a16_counter_count(m, n))
    e.w4a16_gemm_rope_kv(x, blob, out, n, group_size, ws.ws, ws.counters,
                         status_buffer(x.device), positions, cos_sin, slots, k_cache, v_cache,
                         layer, hq, hkv)
    LAUNCHES.add(1)
    return out


def w4a16_plan(m: int, n: int, k: int, splits: int = 0):
    return ext().w4a16_plan(m, n, k, splits)


# ----------------------------------------------------------------- attention
def attn_decode(q, k_cache, v_cache, block_tables, seq_lens, out, layer: int, num_splits: int,
                blocks_per_split: int, part_o, part_ml, scale: float, window: int = 0,
                sinks: int = 0):
    """Paged decode attention; ``window`` > 0: sliding window of that many
    positions (plus the first ``sinks`` positions)."""
    if _dbg.ENABLED and not torch.cuda.is_current_stream_capturing():
        _dbg.check_paged(block_tables, seq_lens, k_cache.shape[1])
    ext().attn_decode(q, k_cache, v_cache, block_tables, seq_lens, out, layer, num_splits,
                      blocks_per_split, part_o, part_ml, scale, status_buffer(q.device), window,
                      sinks)
    LAUNCHES.add(2 if num_splits > 1 else 1)
    return out


def attn_prefill(q, k_cache, v_cache, block_tables, tiles, out, layer: int, scale: float,
                 window: int = 0, sinks: int = 0):
    ext().attn_prefill(q, k_cache, v_cache, block_tables, tiles, out, layer, scale,
                       status_buffer(q.device), window, sinks)
    LAUNCHES.add(1)
    return out


def decode_split_plan(batch: int, kv_heads: int, max_blocks: int, num_sms: int = 148):
    """Split the context so batch*kv_heads*splits fills about two waves of SMs."""
    pairs = max(1, batch * kv_heads)
    want = max(1, math.ceil(2 * num_sms / pairs))
    splits = max(1, min(want, max(1, max_blocks // 4)))
    bps = max(1, math.ceil(max_blocks / splits))
    splits = max(1, math.ceil(max_blocks / bps))
    return splits, bps


def prefill_tiles(q_lens, ctx_lens, device) -> torch.Tensor:
    """Per 64-row query tile: (seq, first packed row, first position, rows)."""
    tiles = []
    row = 0
    for b, (ql, cl) in enumerate(zip(q_lens, ctx_lens)):
        start_pos = cl - ql
        for t0 in range(0, ql, 64):
            tiles.append((b, row + t0, start_pos + t0, min(64, ql - t0)))
        row += ql
    # Longest (most KV) tiles first: better tail behaviour for causal work.
    tiles.sort(key=lambda t: -(t[2] + t[3]))
    if not tiles:
        return torch.zeros(0, 4, dtype=torch.int32, device=device)
    return torch.tensor(tiles, dtype=torch.int32, device=device)


# ----------------------------------------------------------------- small ops
def embedding(ids, table, out, vocab_lo: int = 0):
    if _dbg.ENABLED and not torch.cuda.is_current_stream_capturing():
        _dbg.check_range("token ids", ids, 0, 1 << 31)
    ext().embedding(ids, table, out, vocab_lo)
    LAUNCHES.add(1)
    return out


def rmsnorm(x, w, out, eps: float, residual=None):
    """out = rmsnorm(x + residual) * w; residual (if given) is updated in place."""
    ext().rmsnorm(x, residual, w, out, eps)
    LAUNCHES.add(1)
    return out


def head_rmsnorm(qkv, q_w, k_w, hq, hkv, d, eps):
    """In-place per-head RMSNorm of the q and k heads of a fused qkv row."""
    ext().head_rmsnorm(qkv, q_w, k_w, hq, hkv, d, eps)
    LAUNCHES.add(1)
    return qkv


def rope_kv_write(qkv, positions, cos_sin, slots, k_cache, v_cache, layer, hq, hkv, d, rot,
                  interleaved=False):
    if _dbg.ENABLED and not torch.cuda.is_current_stream_capturing():
        _dbg.check_range("kv slots", slots, 0, k_cache.shape[1] * 16, allow=(-1,))
        _dbg.check_range("positions", positions, 0, cos_sin.shape[0])
    ext().rope_kv_write(qkv, positions, cos_sin, slots, k_cache, v_cache, layer, hq, hkv, d, rot,
                        interleaved)
    LAUNCHES.add(1)


def argmax(logits, out_idx, out_val=None, idx_offset: int = 0):
    ext().argmax(logits, out_idx, out_val, idx_offset)
    LAUNCHES.add(1)
    return out_idx


def sample(logits, params, history, hist_len, work, seeds, offsets, out):
    ext().sample(logits, params, history, hist_len, work, seeds, offsets, out)
    LAUNCHES.add(1)
    return out


def spec_verify(target, draft, out):
    ext().spec_verify(target, draft, out)
    LAUNCHES.add(1)
    return out


_VERIFY_SCRATCH: dict = {}


def spec_verify_fused(logits, row_seq, row_start, draft, kv_len, out, scratch=None):
    """One kernel for a speculative round on a single GPU: argmax of every
    verify row of `logits` [R, V], comparison with `draft` [B, k] (-1
    padded), out [B, k+2] = accepted drafts + correction token, -1 padding,
    count in the last column, and kv_len[b] += count on the device.
    ``scratch`` = (picks int32 [>=R], done int32 [>=B] zeroed; the kernel
    leaves it zeroed): a captured graph passes its own, eager calls share a
    cached pair."""
    R, B = logits.shape[0], draft.shape[0]
    sc = scratch
    if sc is None:
        key = logits.device.index or 0
        sc = _VERIFY_SCRATCH.get(key)
        if sc is None or sc[0].numel() < R or sc[1].numel() < B:
            sc = (torch.empty(max(R, 256), dtype=torch.int32, device=logits.device),
                  torch.zeros(max(B, 64), dtype=torch.int32, device=logits.device))
            _VERIFY_SCRATCH[key] = sc
    ext().spec_verify_fused(logits, row_seq, row_start, draft, sc[0], sc[1], kv_len, out)
    LAUNCHES.add(1)
    return out


# ----------------------------------------------------------------- Gated DeltaNet
def gdn_conv(x, channels: int, w, state, seq_start, block_tables, block_slot):
    """Causal depthwise conv (width 4) + SiLU of x[:, :channels] in place,
    per sequence (token ranges seq_start[b]..seq_start[b+1]), with the conv
    state of each sequence's slot (block_slot[block_tables[b, 0]]) read and
    updated."""
    ext().gdn_conv(x, channels, w, state, seq_start, block_tables, block_slot)
    LAUNCHES.add(1)
    return x


def gdn_recurrent(qkv, z, ab, a_log, dt_bias, norm_w, state, seq_start, block_tables,
                  block_slot, out, hk: int, hv: int, eps: float):
    """Gated delta-rule recurrence of every (sequence, value head) over its
    tokens, fp32 state updated in place, gated RMSNorm of the output fused."""
    ext().gdn_recurrent(qkv, z, ab, a_log, dt_bias, norm_w, state, seq_start, block_tables,
                        block_slot, out, hk, hv, eps)
    LAUNCHES.add(1)
    return out


def sigmoid_gate(x, gate):
    """x *= sigmoid(gate[:, :x.shape[1]]) in place."""
    ext().sigmoid_gate(x, gate)
    LAUNCHES.add(1)
    return x


# ----------------------------------------------------------------- MoE
_GATE_CNT: dict = {}


def _gate_counters(device, n: int) -> torch.Tensor:
    """Per-token completion counters of the gate kernel (zero between
    launches: the kernel resets each one it uses)."""
    key = torch.device(device).index or 0
    buf = _GATE_CNT.get(key)
    if buf is None or buf.numel() < n:
        buf = torch.zeros(max(n, 4096), dtype=torch.int32, device=device)
        _GATE_CNT[key] = buf
    return buf


def moe_topk_gate(x, wg, k: int, scoring: int = 0, norm_topk: bool = True,
                  routed_scale: float = 1.0, bias=None, logits_out=None):
    """Router + top-k: returns (ids int32 [T, k], weights fp32 [T, k])."""
    T = x.shape[0]
    E = wg.shape[0]
    ids = torch.empty(T, k, dtype=torch.int32, device=x.device)
    w = torch.empty(T, k, dtype=torch.float32, device=x.device)
    logits = logits_out if logits_out is not None else torch.empty(
        max(1, T * E), dtype=torch.float32, device=x.device)
    ext().moe_topk_gate(x, wg, bias, k, scoring, norm_topk, routed_scale, ids, w, logits,
                        _gate_counters(x.device, T))
    LAUNCHES.add(1)
    return ids, w


def moe_permute(ids, num_experts: int, x=None):
    """Counting sort of (token, slot) pairs by expert; optionally gathers x."""
    if _dbg.ENABLED and not torch.cuda.is_current_stream_capturing():
        _dbg.check_range("expert ids", ids, 0, num_experts)
    n = ids.numel()
    dev = ids.device
    offsets = torch.empty(num_experts + 1, dtype=torch.int32, device=dev)
    perm = torch.empty(max(1, n), dtype=torch.int32, device=dev)
    inv = torch.empty(max(1, n), dtype=torch.int32, device=dev)
    xp = None
    if x is not None:
        xp = torch.empty(max(1, n), x.shape[1], dtype=x.dtype, device=dev)
    ext().moe_permute(ids, num_experts, offsets, perm, inv, x, xp)
    LAUNCHES.add(2 if x is not None else 1)
    return offsets, perm, inv, xp


def w4a16_gemm_grouped(x, blob, n: int, group_size: int, epilogue: int, offsets,
                       num_groups: int, max_rows: int, out=None, out_rows=None):
    """Grouped (per-expert) W4A16 GEMM.  ``out_rows`` (int64 [rows], optional):
    row m of the result is stored at address out_rows[m] (peer memory for
    expert parallelism) instead of into ``out``."""
    m = x.shape[0]
    n_out = n // 2 if epilogue == EPI_SILU else n
    if out is None:
        out = torch.empty(1 if out_rows is not None else m, n_out, dtype=torch.bfloat16,
                          device=x.device)
    ext().w4a16_gemm_grouped(x, blob, out, n, group_size, epilogue, offsets, num_groups,
                             max_rows, status_buffer(x.device), out_rows)
    LAUNCHES.add(1)
    return out


def moe_prep_fp16(x, rows: int, perm=None, topk: int = 1, rows_dev=None, out=None):
    """Prepared activations for the grouped small-M GEMM: fp16 rows (scaled
    by a power of two per row) and per-k-block offset corrections.  Row r is
    x[perm[r] // topk] when ``perm`` is given (gather into expert order)."""
    K = x.shape[1]
    ld16, lds = ext().moe_prep_shape(K)
    if out is not None:
        x16, xs = out
    else:
        x16 = torch.empty(max(1, rows), ld16, dtype=torch.float16, device=x.device)
        xs = torch.empty(max(1, rows), lds, dtype=torch.float32, device=x.device)
    ext().moe_prep_fp16(x, perm, topk, rows, x16, xs, rows_dev)
    LAUNCHES.add(1)
    return x16, xs


def w4a16_gemv_grouped(x16, xs, blob, n: int, epilogue: int, offsets, num_groups: int,
                       out=None, out_rows=None, sched=None):
    """Grouped small-M W4A16 GEMM (group 128) on prepared activations; the
    decode path of the MoE experts (few rows per expert).  ``sched`` (int32
    [2] zeros, owned by the call site and never used by two launches at
    once) switches the kernel to dynamic unit scheduling."""
    rows = x16.shape[0]
    n_out = n // 2 if epilogue == EPI_SILU else n
    if out is None:
        out = torch.empty(rows, n_out, dtype=torch.bfloat16, device=x16.device)
    ext().w4a16_gemv_grouped(x16, xs, blob, out, n, epilogue, offsets, num_groups,
                             status_buffer(x16.device), out_rows, sched)
    LAUNCHES.add(1)
    return out


def moe_combine(y, inv, w, add=None, out=None, shared=None, shared_gate=None):
    """out[t] = add[t] + sum_j w[t, j] y[inv[t, j]] + g_t * shared[t], with
    g_t = sigmoid(shared_gate[t]) when a gate is given (else 1)."""
    T = w.shape[0]
    if out is None:
        out = torch.empty(T, y.shape[1], dtype=torch.bfloat16, device=y.device)
    ext().moe_combine(y, inv, w, add, out, shared, shared_gate)
    LAUNCHES.add(1)
    return out
