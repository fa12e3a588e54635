"""INT4 formats: canonical packing and the kernel blob layout (CPU)."""
import torch

from cascadia_b200.quant import Int4Weight, interleave_rows, pack_nibbles, unpack_nibbles


def test_pack_unpack_roundtrip():
    g = torch.Generator().manual_seed(0)
    q = torch.randint(0, 16, (16, 64), generator=g, dtype=torch.int32)
    assert torch.equal(unpack_nibbles(pack_nibbles(q)), q)


def test_nibble_order_matches_reference():
    # column 8i+j in bits 4j (crates/cascadia-int4-gemm/src/lib.rs:11-22)
    q = torch.zeros(1, 8, dtype=torch.int32)
    q[0, 1] = 0xA
    q[0, 7] = 0x3
    w = int(pack_nibbles(q)[0, 0]) & 0xFFFFFFFF
    assert w == (0xA << 4) | (0x3 << 28)


def test_quantize_error_bound():
    g = torch.Generator().manual_seed(1)
    w = torch.randn(128, 256, generator=g) * 0.02
    qw = Int4Weight.quantize(w, 128)
    err = (qw.dequant_bf16().float() - w).abs()
    s = qw.scales.float().repeat_interleave(128, 1)
    assert bool((err <= s * 0.53 + 1e-6).all())


def _decode_blob(blob, n, k, gs, interleave):
    """Read the blob the way the GEMM kernel does and return bf16 [N, K]."""
    rt, kb = n // 128, k // 128
    per = 8192 + 128 * (128 // gs) * 2
    b = blob.view(rt, kb, per)
    out = torch.zeros(n, k, dtype=torch.float32)
    for r in range(rt):
        for c in range(kb):
            blk = b[r, c]
            phys = blk[:8192].contiguous().view(torch.int32).view(128, 4, 4)
            rows = torch.arange(128)
            # undo the chunk swizzle: logical chunk c lives at c ^ ((r >> 1) & 3)
            logical = torch.stack([phys[rows, (c ^ ((rows >> 1) & 3))] for c in range(4)], 1)
            words = logical.reshape(128, 16).to(torch.int64) & 0xFFFFFFFF
            sc = blk[8192:].contiguous().view(torch.bfloat16).view(128, 128 // gs).float()
            vals = torch.zeros(128, 128)
            for wi in range(16):
                w = words[:, wi]
                for h in range(4):
                    lo = (w >> (4 * h)) & 0xF
                    hi = (w >> (16 + 4 * h)) & 0xF
                    vals[:, wi * 8 + 2 * h] = lo.float()
                    vals[:, wi * 8 + 2 * h + 1] = hi.float()
            s = sc.repeat_interleave(gs, 1)
            deq = ((vals - 8.0).to(torch.bfloat16).float() * s).to(torch.bfloat16).float()
            out[r * 128:(r + 1) * 128, c * 128:(c + 1) * 128] = deq
    return out


def test_blob_layout_matches_dequant():
    for gs in (128, 32):
        g = torch.Generator().manual_seed(2)
        qw = Int4Weight.random(256, 256, group_size=gs, generator=g)
        blob = qw.blob()
        dec = _decode_blob(blob, 256, 256, gs, False)
        assert torch.equal(dec, qw.dequant_bf16().float())


def test_blob_gate_up_interleave():
    g = torch.Generator().manual_seed(3)
    qw = Int4Weight.random(256, 128, generator=g)  # [gate(128); up(128)]
    dec = _decode_blob(qw.blob(interleave_gate_up=True), 256, 128, 128, True)
    ref = interleave_rows(qw.dequant_bf16().float())
    assert torch.equal(dec, ref)


def test_debug_index_checks():
    import pytest
    import torch

    from cascadia_b200.ops import debug

    debug.check_range("ok", torch.tensor([0, 3, -1]), 0, 4, allow=(-1,))
    with pytest.raises(debug.IndexCheckError):
        debug.check_range("bad", torch.tensor([0, 4]), 0, 4)
    debug.check_paged(torch.tensor([[2, 5, 0]]), torch.tensor([20]), 8)
    with pytest.raises(debug.IndexCheckError):
        debug.check_paged(torch.tensor([[2, 9, 0]]), torch.tensor([20]), 8)
    with pytest.raises(debug.IndexCheckError):
        debug.check_paged(torch.tensor([[2, 5]]), torch.tensor([40]), 8)
