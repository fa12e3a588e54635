"""Failure detection on the GPU without a GPU fault: a peer that never
signals.  One kernel waits on a flag that nothing sets; its bounded wait
(2 s of %globaltimer) must run out, record the peer-timeout status code in
the device status word, leave the kernel normally and keep the context
usable.  Single GPU, single launch, no second rank."""
import time

import pytest
import torch

from cascadia_b200 import ops

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
PEER_TIMEOUT = 301


def test_fused_allreduce_times_out_on_a_silent_peer():
    H, M = 256, 4
    ops.read_status(DEV)  # clear
    bufs = [torch.zeros(M, H, dtype=torch.bfloat16, device=DEV) for _ in range(2)]
    sigs = [torch.zeros(8, dtype=torch.int32, device=DEV) for _ in range(2)]
    epoch = torch.zeros(1, dtype=torch.int32, device=DEV)
    done = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = torch.empty(M, H, dtype=torch.bfloat16, device=DEV)
    bp = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64)
    sp = torch.tensor([s.data_ptr() for s in sigs], dtype=torch.int64)
    t0 = time.time()
    # rank 0 of a 2-rank group whose rank 1 never runs
    # (plain peer loads: mc_ptr 0, no multicast object is involved)
    ops.ext().ar_rmsnorm(bp, 0, sp, epoch, done, ops.status_buffer(DEV), 0, 2, M, H, None,
                         None, out, 1e-5, 0)
    torch.cuda.synchronize()
    assert time.time() - t0 < 30
    assert ops.read_status(DEV) == PEER_TIMEOUT
    # The context still works.
    x = torch.ones(8, device=DEV)
    assert float((x * 2).sum()) == 16.0
    assert ops.read_status(DEV) == 0


def test_expert_combine_times_out_when_results_never_return():
    H, T, k, E = 256, 3, 2, 8
    ops.read_status(DEV)
    W, cap = 2, 64
    xbuf = torch.zeros(W * cap * H, dtype=torch.bfloat16, device=DEV)
    rbuf = torch.zeros(W * cap * H, dtype=torch.bfloat16, device=DEV)
    meta = torch.zeros(W * cap, dtype=torch.int32, device=DEV)
    sig = torch.zeros(64, dtype=torch.int32, device=DEV)
    other_sig = torch.zeros(64, dtype=torch.int32, device=DEV)
    ptr = lambda t, u: torch.tensor([t.data_ptr(), u.data_ptr()], dtype=torch.int64)  # noqa: E731
    epoch = torch.zeros(1, dtype=torch.int32, device=DEV)
    done = torch.zeros(1, dtype=torch.int32, device=DEV)
    dest = torch.zeros(T * k, dtype=torch.int32, device=DEV)
    pos = torch.arange(T * k, dtype=torch.int32, device=DEV)
    w = torch.full((T, k), 0.5, device=DEV)
    add = torch.ones(T, H, dtype=torch.bfloat16, device=DEV)
    out = torch.empty(T, H, dtype=torch.bfloat16, device=DEV)
    # No rank ever raises the "returned" flags: the combine must give up.
    ops.ext().ep_combine(w, dest, pos, add, out, ptr(xbuf, xbuf), ptr(rbuf, rbuf),
                         ptr(meta, meta), ptr(sig, other_sig), epoch, done,
                         ops.status_buffer(DEV), 0, W, cap, E // W)
    torch.cuda.synchronize()
    assert ops.read_status(DEV) == PEER_TIMEOUT
    assert torch.equal(out, add)  # nothing combined, residual passed through
