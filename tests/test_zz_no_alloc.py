"""The allocation-free W4A16 GEMM entry point, called through its exported C
symbol, against the regular entry point (the same kernel choice: small-M up
to 8 rows, split-K tcgen05 above; caller workspace).

Collected last (file name) so that it also runs after every other test in
one process; it must pass alone in a fresh process too.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

OK, EINVAL, ETOOBIG = 0, 1, 2
MAX_WS_FLOATS = 6 << 20


def _lib():
    from cascadia_b200 import _C

    lib = ctypes.CDLL(_C.__file__)
    f = lib.cb_w4a16_gemm_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, ctypes.c_longlong, ctypes.c_void_p, ctypes.c_void_p,
                  ctypes.c_longlong, ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int,
                  ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                  ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int]
    return f


def _call(f, x, blob, out, residual, n, gs, epi, status=None):
    err = ctypes.create_string_buffer(512)
    rc = f(x.data_ptr(), x.stride(0), blob.data_ptr(), out.data_ptr(), out.stride(0),
           residual.data_ptr() if residual is not None else None,
           residual.stride(0) if residual is not None else 0,
           x.shape[0], n, x.shape[1], gs, epi,
           status.data_ptr() if status is not None else None,
           torch.cuda.current_stream().cuda_stream, err, len(err))
    return rc, err.value.decode()


@pytest.mark.parametrize("m,n,k,gs,epi", [
    (16, 4096, 4096, 128, 0),    # split-K over several k-ranges (scratch partials + counters)
    (5, 2048, 14336, 128, 2),    # small-M kernel + residual epilogue
    (33, 1024, 2048, 32, 1),     # group 32, SiLU(gate)*up epilogue
    (64, 6144, 4096, 128, 0),
    (96, 4096, 4096, 128, 2),    # split-K tcgen05 kernel, residual epilogue
])
def test_noalloc_matches_regular_entry_point(m, n, k, gs, epi):
    from cascadia_b200 import ops
    from cascadia_b200.quant import Int4Weight

    dev = torch.device("cuda")
    f = _lib()
    g = torch.Generator().manual_seed(m * 7 + n)
    w = Int4Weight.random(n, k, 0.05, gs, generator=g)
    blob = w.to(dev).blob(interleave_gate_up=(epi == 1))
    n_out = n // 2 if epi == 1 else n
    residual = (torch.randn(m, n, generator=g) * 0.5).to(torch.bfloat16).to(dev) \
        if epi == 2 else None
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    for call in range(2):
        x = (torch.randn(m, k, generator=g) * 0.5).to(torch.bfloat16).to(dev)
        want = ops.w4a16_gemm(x, blob, n, gs, epi, residual)
        got = torch.full((m, n_out), float("nan"), dtype=torch.bfloat16, device=dev)
        rc, msg = _call(f, x, blob, got, residual, n, gs, epi, status if call else None)
        assert rc == OK, msg
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert ops.read_status(dev) == 0
        scale = want.float().abs().max().item()
        err = (got.float() - want.float()).abs().max().item()
        assert err <= 0.02 * scale + 1e-2, (call, err, scale)


def test_noalloc_rejects_oversized_and_bad_shapes():
    from cascadia_b200 import ops
    from cascadia_b200.quant import blob_bytes

    dev = torch.device("cuda")
    f = _lib()
    # Invalid arguments are rejected before any launch.
    x2 = torch.zeros(4, 100, dtype=torch.bfloat16, device=dev)
    out2 = torch.zeros(4, 256, dtype=torch.bfloat16, device=dev)
    blob2 = torch.zeros(blob_bytes(256, 128, 128), dtype=torch.uint8, device=dev)
    rc, msg = _call(f, x2, blob2, out2, None, 256, 128, 0)
    assert rc == EINVAL and "invalid argument" in msg
    # A shape whose scratch exceeds the fixed maximum, found with the same
    # planner the entry point uses (the regular entry point's workspace
    # query).  The smallest such weight is allocated in full, so that even a
    # wrong prediction could only run a kernel on a real (zero) weight.
    cands = []
    for m in (1, 2, 4, 8):
        for n in (65536, 262144):
            for k in (16384, 65536):
                if ops.ext().w4a16_workspace_floats(m, n, k, 0) > MAX_WS_FLOATS:
                    cands.append((n * k, m, n, k))
    if not cands:
        pytest.skip("no shape of the current planner needs more than the fixed scratch")
    _, m, n, k = min(cands)
    x = torch.zeros(m, k, dtype=torch.bfloat16, device=dev)
    blob = torch.zeros(blob_bytes(n, k, 128), dtype=torch.uint8, device=dev)
    out = torch.zeros(m, n, dtype=torch.bfloat16, device=dev)
    rc, msg = _call(f, x, blob, out, None, n, 128, 0)
    torch.cuda.synchronize()
    assert rc == ETOOBIG and "fixed maximum" in msg, (m, n, k, rc, msg)
    del blob
