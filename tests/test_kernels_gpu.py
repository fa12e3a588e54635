"""Numerics of every sm_100a kernel against a plain PyTorch fp32 reference."""
import math

import pytest
import torch

from cascadia_b200 import ops
from cascadia_b200.ops import reference as ref
from cascadia_b200.quant import Int4Weight, interleave_rows

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _close(out, expect, rtol=2e-2, atol=2e-2):
    out = out.float().cpu()
    expect = expect.float().cpu()
    err = (out - expect).abs()
    tol = atol + rtol * expect.abs()
    bad = (err > tol).sum().item()
    assert bad == 0, f"{bad} mismatches, max err {err.max().item():.4g}"


def _status_ok():
    assert ops.read_status(torch.device(DEV)) == 0, "device status word set (timeout)"


@pytest.mark.parametrize("m", [1, 5, 16, 33, 64, 130, 300])
@pytest.mark.parametrize("gs", [128, 32])
def test_w4a16_gemm_store(m, gs):
    g = torch.Generator().manual_seed(m * 7 + gs)
    n, k = 384, 1024
    qw = Int4Weight.random(n, k, group_size=gs, generator=g, std=0.05)
    x = (torch.randn(m, k, generator=g) * 0.5).to(torch.bfloat16)
    blob = qw.blob().to(DEV)
    y = ops.w4a16_gemm(x.to(DEV), blob, n, group_size=gs)
    torch.cuda.synchronize()
    _status_ok()
    expect = x.float() @ qw.dequant_bf16().float().t()
    _close(y, expect, rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("splits", [1, 2, 3, 8])
def test_w4a16_gemm_splitk_deterministic(splits):
    g = torch.Generator().manual_seed(11)
    n, k, m = 256, 2048, 24
    qw = Int4Weight.random(n, k, generator=g, std=0.05)
    x = (torch.randn(m, k, generator=g)).to(torch.bfloat16).to(DEV)
    blob = qw.blob().to(DEV)
    y1 = ops.w4a16_gemm(x, blob, n, splits=splits)
    y2 = ops.w4a16_gemm(x, blob, n, splits=splits)
    torch.cuda.synchronize()
    _status_ok()
    assert torch.equal(y1, y2)
    expect = x.float().cpu() @ qw.dequant_bf16().float().t()
    _close(y1, expect, rtol=1e-2, atol=2e-2)


@pytest.mark.parametrize("m", [3, 64])
def test_w4a16_gemm_silu(m):
    g = torch.Generator().manual_seed(5)
    inter, k = 256, 512
    qw = Int4Weight.random(2 * inter, k, generator=g, std=0.05)  # [gate; up]
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    blob = qw.blob(interleave_gate_up=True).to(DEV)
    y = ops.w4a16_gemm(x.to(DEV), blob, 2 * inter, epilogue=ops.EPI_SILU)
    torch.cuda.synchronize()
    _status_ok()
    full = x.float() @ qw.dequant_bf16().float().t()
    expect = ref.silu_mul(full[:, :inter], full[:, inter:])
    _close(y, expect)


@pytest.mark.parametrize("m", [2, 40])
def test_w4a16_gemm_residual(m):
    g = torch.Generator().manual_seed(9)
    n, k = 512, 768
    qw = Int4Weight.random(n, k, generator=g, std=0.05)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    r = torch.randn(m, n, generator=g).to(torch.bfloat16)
    rd = r.to(DEV)
    y = ops.w4a16_gemm(x.to(DEV), qw.blob().to(DEV), n, epilogue=ops.EPI_RESID, residual=rd,
                       out=rd)
    torch.cuda.synchronize()
    _status_ok()
    expect = x.float() @ qw.dequant_bf16().float().t() + r.float()
    _close(y, expect)


@pytest.mark.parametrize("m", [1, 3, 8, 9, 16])
@pytest.mark.parametrize("gs", [128, 32])
@pytest.mark.parametrize("epi", [0, 1, 2])
@pytest.mark.parametrize("n,k", [(384, 1024), (256, 14336)])
def test_w4a16_gemv_small_m(m, gs, epi, n, k):
    """The small-M kernel (warp MMAs fed straight from registers) against the
    fp32 reference, for every epilogue, with and without split-K."""
    g = torch.Generator().manual_seed(m * 131 + gs + epi + k)
    qw = Int4Weight.random(n, k, group_size=gs, generator=g, std=0.05)
    x = (torch.randn(m, k, generator=g) * 0.5).to(torch.bfloat16)
    r = torch.randn(m, n, generator=g).to(torch.bfloat16)
    blob = qw.blob(interleave_gate_up=(epi == ops.EPI_SILU)).to(DEV)
    e = ops.ext()
    ws = ops.default_workspace(torch.device(DEV))
    ws.ensure(e.gemv_workspace_floats(m, n, k, 0), n // 128)
    n_out = n // 2 if epi == ops.EPI_SILU else n
    out = torch.full((m, n_out), float("nan"), dtype=torch.bfloat16, device=DEV)
    rd = r.to(DEV) if epi == ops.EPI_RESID else None
    for _ in range(2):  # twice: the split-K counters must come back to zero
        e.w4a16_gemv(x.to(DEV), blob, out, n, gs, epi, rd, ws.ws, ws.counters,
                     ops.status_buffer(torch.device(DEV)), 0)
    torch.cuda.synchronize()
    _status_ok()
    # Group 128 applies the scale in fp32 after the k-block sum (no bf16
    # rounding of (q-8)*scale): compare against the exact fp32 dequant.
    if gs == 128:
        wq = (qw.unpack().float() - 8.0) * qw.scales.float().repeat_interleave(gs, dim=1)
    else:
        wq = qw.dequant_bf16().float()
    full = x.float() @ wq.t()
    if epi == ops.EPI_SILU:
        expect = ref.silu_mul(full[:, :n // 2], full[:, n // 2:])
    elif epi == ops.EPI_RESID:
        expect = full + r.float()
    else:
        expect = full
    _close(out, expect, rtol=1e-2, atol=2e-2)


def test_gemv_and_tcgen05_paths_agree():
    g = torch.Generator().manual_seed(3)
    n, k, m = 1024, 4096, 5
    qw = Int4Weight.random(n, k, generator=g, std=0.05)
    x = (torch.randn(m, k, generator=g) * 0.5).to(torch.bfloat16).to(DEV)
    blob = qw.blob().to(DEV)
    y_small = ops.w4a16_gemm(x, blob, n)            # small-M path (M <= 8)
    y_tc = ops.w4a16_gemm(x, blob, n, splits=4)     # forced splits: tcgen05 path
    torch.cuda.synchronize()
    _status_ok()
    _close(y_small, y_tc.float(), rtol=1e-2, atol=1e-2)


def test_rmsnorm_and_residual():
    g = torch.Generator().manual_seed(3)
    for h in (2048, 4096, 7168):
        x = torch.randn(5, h, generator=g).to(torch.bfloat16)
        r = torch.randn(5, h, generator=g).to(torch.bfloat16)
        w = (1 + 0.1 * torch.randn(h, generator=g)).to(torch.bfloat16)
        out = torch.empty(5, h, dtype=torch.bfloat16, device=DEV)
        ops.rmsnorm(x.to(DEV), w.to(DEV), out, 1e-5)
        _close(out, ref.rmsnorm(x, w, 1e-5))
        rd = r.to(DEV)
        ops.rmsnorm(x.to(DEV), w.to(DEV), out, 1e-5, residual=rd)
        s = (x.float() + r.float()).to(torch.bfloat16)
        _close(rd, s, rtol=0, atol=0)
        _close(out, ref.rmsnorm(s, w, 1e-5))


def _rope_table(max_pos, rot, theta=500000.0):
    inv = 1.0 / (theta ** (torch.arange(0, rot, 2).float() / rot))
    f = torch.outer(torch.arange(max_pos).float(), inv)
    return torch.cat([f.cos(), f.sin()], dim=1)


def test_rope_kv_write():
    g = torch.Generator().manual_seed(4)
    hq, hkv, d, t, nb, layers = 8, 2, 128, 7, 6, 2
    qkv = torch.randn(t, (hq + 2 * hkv) * d, generator=g).to(torch.bfloat16)
    pos = torch.tensor([0, 1, 2, 17, 40, 41, 63], dtype=torch.int32)
    slots = torch.tensor([0, 1, 2, 17, 40, 41, -1], dtype=torch.int32)
    cs = _rope_table(128, d)
    kc = torch.zeros(layers, nb, hkv, 16, d, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    q_dev = qkv.to(DEV)
    ops.rope_kv_write(q_dev, pos.to(DEV), cs.to(DEV), slots.to(DEV), kc, vc, 1, hq, hkv, d, d)
    torch.cuda.synchronize()
    qf = qkv.float().view(t, hq + 2 * hkv, d)
    q_ref = ref.apply_rope(qf[:, :hq], pos, cs, d)
    k_ref = ref.apply_rope(qf[:, hq:hq + hkv], pos, cs, d)
    _close(q_dev.view(t, -1, d)[:, :hq], q_ref)
    for i in range(t):
        s = int(slots[i])
        if s < 0:
            continue
        _close(kc[1, s // 16, :, s % 16], k_ref[i])
        _close(vc[1, s // 16, :, s % 16], qf[i, hq + hkv:], rtol=0, atol=0)
    assert kc[0].abs().sum().item() == 0


def _make_cache(seq_lens, hkv, d, layers, layer, g, nb_extra=3):
    """Random K/V in a shuffled paged cache; returns caches, tables, dense copies."""
    bs = len(seq_lens)
    blocks = [(l + 15) // 16 for l in seq_lens]
    nb = sum(blocks) + nb_extra
    perm = torch.randperm(nb, generator=g)
    kc = torch.randn(layers, nb, hkv, 16, d, generator=g).to(torch.bfloat16)
    vc = torch.randn(layers, nb, hkv, 16, d, generator=g).to(torch.bfloat16)
    maxb = max(blocks)
    table = torch.zeros(bs, maxb + 2, dtype=torch.int32)
    dense = []
    c = 0
    for b in range(bs):
        ids = perm[c:c + blocks[b]]
        c += blocks[b]
        table[b, :blocks[b]] = ids.to(torch.int32)
        k = kc[layer, ids].permute(0, 2, 1, 3).reshape(-1, hkv, d)[:seq_lens[b]]
        v = vc[layer, ids].permute(0, 2, 1, 3).reshape(-1, hkv, d)[:seq_lens[b]]
        dense.append((k, v))
    return kc, vc, table, dense


@pytest.mark.parametrize("d,hq,hkv", [(128, 32, 8), (64, 32, 8), (128, 16, 1), (256, 16, 2),
                                      (256, 4, 2), (512, 8, 2), (512, 16, 1)])
@pytest.mark.parametrize("splits", [1, 3])
def test_attn_decode(d, hq, hkv, splits):
    g = torch.Generator().manual_seed(d + hq + splits)
    seq_lens = [1, 16, 17, 100, 300]
    layers, layer = 2, 1
    kc, vc, table, dense = _make_cache(seq_lens, hkv, d, layers, layer, g)
    bs = len(seq_lens)
    q = torch.randn(bs, hq * d, generator=g).to(torch.bfloat16)
    maxb = table.shape[1]
    bps = max(1, math.ceil(maxb / splits))
    sp = max(1, math.ceil(maxb / bps))
    g_ = hq // hkv
    part_o = torch.empty(bs * hkv * sp * g_ * d, dtype=torch.float32, device=DEV)
    part_ml = torch.empty(bs * hkv * sp * g_ * 2, dtype=torch.float32, device=DEV)
    out = torch.empty(bs, hq * d, dtype=torch.bfloat16, device=DEV)
    scale = 1.0 / math.sqrt(d)
    ops.attn_decode(q.to(DEV), kc.to(DEV), vc.to(DEV), table.to(DEV),
                    torch.tensor(seq_lens, dtype=torch.int32, device=DEV), out, layer, sp, bps,
                    part_o, part_ml, scale)
    torch.cuda.synchronize()
    _status_ok()
    for b in range(bs):
        k, v = dense[b]
        e = ref.attention(q[b].view(1, hq, d), k, v, torch.tensor([seq_lens[b] - 1]), scale)
        _close(out[b].view(hq, d), e[0], rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("d", [128, 64, 256])
def test_attn_prefill(d):
    g = torch.Generator().manual_seed(21 + d)
    hq, hkv = 8, 2
    ctx = [5, 64, 130, 257]
    qlen = [5, 64, 70, 100]  # last two have a cached prefix (chunked prefill)
    layers, layer = 1, 0
    kc, vc, table, dense = _make_cache(ctx, hkv, d, layers, layer, g)
    t = sum(qlen)
    q = torch.randn(t, hq * d, generator=g).to(torch.bfloat16)
    tiles = ops.prefill_tiles(qlen, ctx, DEV)
    out = torch.zeros(t, hq * d, dtype=torch.bfloat16, device=DEV)
    scale = 1.0 / math.sqrt(d)
    ops.attn_prefill(q.to(DEV), kc.to(DEV), vc.to(DEV), table.to(DEV), tiles, out, layer, scale)
    torch.cuda.synchronize()
    _status_ok()
    row = 0
    for b in range(len(ctx)):
        k, v = dense[b]
        pos = torch.arange(ctx[b] - qlen[b], ctx[b])
        e = ref.attention(q[row:row + qlen[b]].view(-1, hq, d), k, v, pos, scale)
        _close(out[row:row + qlen[b]].view(-1, hq, d), e, rtol=2e-2, atol=2e-2)
        row += qlen[b]


def test_embedding_argmax():
    g = torch.Generator().manual_seed(6)
    table = torch.randn(1000, 256, generator=g).to(torch.bfloat16)
    ids = torch.tensor([3, 999, 0, 3], dtype=torch.int32)
    out = torch.empty(4, 256, dtype=torch.bfloat16, device=DEV)
    ops.embedding(ids.to(DEV), table.to(DEV), out)
    _close(out, table[ids.long()], rtol=0, atol=0)
    logits = torch.randn(6, 128256, generator=g)
    logits[2, 77] = 100.0
    logits[3, 5] = logits[3, 9] = 50.0  # tie -> lowest index
    idx = torch.empty(6, dtype=torch.int32, device=DEV)
    ops.argmax(logits.to(DEV), idx)
    exp = ref.argmax(logits)
    assert torch.equal(idx.cpu(), exp)
    assert int(idx[3]) == 5
    lb = logits.to(torch.bfloat16)
    ops.argmax(lb.to(DEV), idx)
    assert torch.equal(idx.cpu(), ref.argmax(lb.float()))


def test_sampling_kernel():
    g = torch.Generator().manual_seed(8)
    m, v = 4, 5000
    logits = torch.randn(m, v, generator=g) * 3
    params = torch.zeros(m, 8)
    params[0] = torch.tensor([0.0, 1.0, 0, 0, 0, 1.0, 0, 0])     # greedy
    params[1] = torch.tensor([1.0, 1.0, 1, 0, 0, 1.0, 0, 0])     # top-k 1 == greedy
    params[2] = torch.tensor([0.7, 0.9, 50, 0, 0, 1.0, 0, 0])    # top-k + top-p
    params[3] = torch.tensor([1.0, 1.0, 0, 0.5, 0.5, 1.3, 0, 0])  # penalties
    hist = torch.tensor([[1, 2, 3, 3], [0, 0, 0, 0], [5, 6, 7, 8], [10, 11, 10, 12]],
                        dtype=torch.int32)
    hl = torch.tensor([4, 0, 4, 4], dtype=torch.int32)
    work = torch.empty(m * v, dtype=torch.float32, device=DEV)
    out = torch.empty(m, dtype=torch.int32, device=DEV)
    seeds = torch.arange(m, dtype=torch.int64, device=DEV) + 123
    offs = torch.zeros(m, dtype=torch.int64, device=DEV)
    ops.sample(logits.to(DEV), params.to(DEV), hist.to(DEV), hl.to(DEV), work, seeds, offs, out)
    torch.cuda.synchronize()
    o = out.cpu()
    pen0 = ref.apply_penalties(logits[0], hist[0].tolist(), 1.0, 0, 0.0, 0.0)
    assert int(o[0]) == int(torch.argmax(pen0))
    assert int(o[1]) == int(torch.argmax(logits[1]))
    # top-k/top-p: sampled token must be inside the kept set.
    p = torch.softmax(logits[2] / 0.7, 0)
    top = torch.argsort(p, descending=True)[:50]
    assert int(o[2]) in set(top.tolist())
    assert 0 <= int(o[3]) < v
    # Distribution check: many draws of a tiny vocab follow the softmax.
    lv = torch.tensor([[0.0, 1.0, 2.0, 3.0]]).repeat(4096, 1)
    pr = torch.tensor([[1.0, 1.0, 0, 0, 0, 1.0, 0, 0]]).repeat(4096, 1)
    out2 = torch.empty(4096, dtype=torch.int32, device=DEV)
    work2 = torch.empty(4096 * 4, dtype=torch.float32, device=DEV)
    seeds2 = torch.arange(4096, dtype=torch.int64, device=DEV)
    ops.sample(lv.to(DEV), pr.to(DEV), None, None, work2, seeds2,
               torch.zeros(4096, dtype=torch.int64, device=DEV), out2)
    freq = torch.bincount(out2.cpu().long(), minlength=4).float() / 4096
    expect = torch.softmax(torch.tensor([0.0, 1.0, 2.0, 3.0]), 0)
    assert (freq - expect).abs().max() < 0.03


def test_spec_verify():
    target = torch.tensor([[5, 6, 7, 8, 9], [1, 2, 3, 4, 5], [9, 9, 9, 9, 9]], dtype=torch.int32)
    draft = torch.tensor([[5, 6, 0, 8], [1, 2, 3, 4], [0, 0, 0, 0]], dtype=torch.int32)
    out = torch.empty(3, 6, dtype=torch.int32, device=DEV)
    ops.spec_verify(target.to(DEV), draft.to(DEV), out)
    o = out.cpu()
    assert o[0, :3].tolist() == [5, 6, 7] and int(o[0, 5]) == 3
    assert o[1, :5].tolist() == [1, 2, 3, 4, 5] and int(o[1, 5]) == 5
    assert int(o[2, 0]) == 9 and int(o[2, 5]) == 1
    for b in range(3):
        r = ref.spec_verify(target[b].tolist(), draft[b].tolist())
        assert o[b, :len(r)].tolist() == r


@pytest.mark.parametrize("d", [128, 256])
@pytest.mark.parametrize("window,sinks", [(40, 0), (70, 4), (16, 20)])
def test_attn_sliding_window_decode_and_prefill(d, window, sinks):
    g = torch.Generator().manual_seed(window + sinks + d)
    hq, hkv = 8, 2
    seq_lens = [1, 30, 100, 257]
    layers, layer = 1, 0
    kc, vc, table, dense = _make_cache(seq_lens, hkv, d, layers, layer, g)
    bs = len(seq_lens)
    scale = 1.0 / math.sqrt(d)
    q = torch.randn(bs, hq * d, generator=g).to(torch.bfloat16)
    maxb = table.shape[1]
    for splits in (1, 3):
        bps = max(1, math.ceil(maxb / splits))
        sp = max(1, math.ceil(maxb / bps))
        part_o = torch.empty(bs * hkv * sp * (hq // hkv) * d, dtype=torch.float32, device=DEV)
        part_ml = torch.empty(bs * hkv * sp * (hq // hkv) * 2, dtype=torch.float32, device=DEV)
        out = torch.empty(bs, hq * d, dtype=torch.bfloat16, device=DEV)
        ops.attn_decode(q.to(DEV), kc.to(DEV), vc.to(DEV), table.to(DEV),
                        torch.tensor(seq_lens, dtype=torch.int32, device=DEV), out, layer, sp, bps,
                        part_o, part_ml, scale, window=window, sinks=sinks)
        torch.cuda.synchronize()
        _status_ok()
        for b in range(bs):
            k, v = dense[b]
            e = ref.attention(q[b].view(1, hq, d), k, v, torch.tensor([seq_lens[b] - 1]), scale,
                              window, sinks)
            _close(out[b].view(hq, d), e[0], rtol=2e-2, atol=2e-2)
    # Prefill: whole prompts and a chunk with a cached prefix.
    qlen = [1, 30, 60, 200]
    t = sum(qlen)
    qp = torch.randn(t, hq * d, generator=g).to(torch.bfloat16)
    tiles = ops.prefill_tiles(qlen, seq_lens, DEV)
    out = torch.zeros(t, hq * d, dtype=torch.bfloat16, device=DEV)
    ops.attn_prefill(qp.to(DEV), kc.to(DEV), vc.to(DEV), table.to(DEV), tiles, out, layer, scale,
                     window=window, sinks=sinks)
    torch.cuda.synchronize()
    _status_ok()
    row = 0
    for b in range(bs):
        k, v = dense[b]
        pos = torch.arange(seq_lens[b] - qlen[b], seq_lens[b])
        e = ref.attention(qp[row:row + qlen[b]].view(-1, hq, d), k, v, pos, scale, window, sinks)
        _close(out[row:row + qlen[b]].view(-1, hq, d), e, rtol=2e-2, atol=2e-2)
        row += qlen[b]


@pytest.mark.parametrize("lens", [[5], [1, 5, 3], [2, 2, 2, 2, 5, 1]])
def test_spec_verify_fused(lens):
    """Fused verify (argmax of every row + accept + correction + KV length)
    against the row-wise argmax and the CPU reference rule."""
    g = torch.Generator().manual_seed(sum(lens))
    V = 1000
    R, B, k = sum(lens), len(lens), max(lens) - 1
    logits = (torch.randn(R, V, generator=g) * 3).to(torch.bfloat16)
    picks = logits.float().argmax(-1)
    offs = [0]
    for n in lens:
        offs.append(offs[-1] + n)
    drafts = []
    for b, n in enumerate(lens):
        # Plant matches for a prefix of random length, then a mismatch.
        d = [int(picks[offs[b] + i]) for i in range(n - 1)]
        cut = int(torch.randint(0, n, (1,), generator=g))
        if cut < n - 1:
            d[cut] = (d[cut] + 1) % V
        drafts.append(d)
    dr = torch.full((B, max(k, 1)), -1, dtype=torch.int32)
    for b, d in enumerate(drafts):
        dr[b, :len(d)] = torch.tensor(d, dtype=torch.int32)
    row_seq = torch.repeat_interleave(torch.arange(B, dtype=torch.int32),
                                      torch.tensor(lens)).to(DEV)
    kv = torch.tensor([100 + 10 * b for b in range(B)], dtype=torch.int32, device=DEV)
    out = torch.empty(B, dr.shape[1] + 2, dtype=torch.int32, device=DEV)
    for _ in range(2):  # twice: the per-sequence counters must reset
        kv_run = kv.clone()
        ops.spec_verify_fused(logits.to(DEV), row_seq, torch.tensor(offs, dtype=torch.int32,
                                                                    device=DEV),
                              dr.to(DEV), kv_run, out)
        torch.cuda.synchronize()
        _status_ok()
        o = out.cpu()
        for b, n in enumerate(lens):
            want = ref.spec_verify([int(picks[offs[b] + i]) for i in range(n)], drafts[b])
            cnt = int(o[b, -1])
            assert o[b, :cnt].tolist() == want
            assert int(kv_run[b]) == 100 + 10 * b + cnt
