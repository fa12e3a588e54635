"""MLA decode-attention microbenchmark (Kimi-K2 shape: 64 heads, latent 512,
rope 64) over the paged latent cache.

    python bench/bench_mla.py [--batch 16] [--ctx 4096] [--layers 4] [--reps 20]

Each call reads every sequence's latent rows of one layer; calls rotate over
`--layers` layers so the cache read (batch x ctx x 1152 bytes per layer)
comes from HBM, not L2.  Timed with CUDA events around a CUDA graph of the
calls; reports the HBM fraction against MEASURED_PEAKS.json.
"""
import argparse
import json
import math
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import torch  # noqa: E402

from cascadia_b200 import ops  # noqa: E402
from cascadia_b200.models.mla import mla_split_plan  # noqa: E402


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--batch", type=int, default=16)
    p.add_argument("--ctx", type=int, default=4096)
    p.add_argument("--heads", type=int, default=64)
    p.add_argument("--layers", type=int, default=4)
    p.add_argument("--reps", type=int, default=20)
    p.add_argument("--splits", type=int, default=0, help="context splits (0: the planner's)")
    a = p.parse_args()
    dev = torch.device("cuda")
    B, C, H, L = a.batch, a.ctx, a.heads, a.layers
    nb = -(-C // 16)
    cache = (torch.randn(L, B * nb, 16, 576, device=dev) * 0.5).to(torch.bfloat16)
    bt = torch.arange(B * nb, dtype=torch.int32, device=dev).view(B, nb)
    lens = torch.full((B,), C, dtype=torch.int32, device=dev)
    q = (torch.randn(B, H, 576, device=dev) * 0.5).to(torch.bfloat16)
    out = torch.empty(B, H, 512, dtype=torch.bfloat16, device=dev)
    splits, bps = mla_split_plan(B, H, nb)
    if a.splits > 0:
        splits, bps = a.splits, -(-nb // a.splits)
    part_o = torch.empty(B * H * splits * 512, dtype=torch.float32, device=dev)
    part_ml = torch.empty(B * H * splits * 2, dtype=torch.float32, device=dev)
    st = ops.status_buffer(dev)

    def run(i):
        ops.ext().mla_decode(q, cache, bt, lens, out, i % L, splits, bps, part_o, part_ml,
                             1.0 / math.sqrt(192), st)

    for i in range(3):
        run(i)
    torch.cuda.synchronize()
    if a.reps > 1:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for i in range(a.reps):
                run(i)
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1000 / a.reps
    else:
        us = float("nan")
    peak = 6543.4
    pk = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                      "MEASURED_PEAKS.json")
    if os.path.exists(pk):
        peak = json.load(open(pk)).get("hbm_gbs", peak)
    nbytes = B * C * 1152 + B * H * (576 + 512) * 2
    print(json.dumps({"kernel": "mla_decode", "batch": B, "ctx": C, "heads": H,
                      "splits": splits, "us": round(us, 2),
                      "GBps": round(nbytes / us / 1e3, 1),
                      "frac_of_measured_hbm": round(nbytes / us / 1e3 / peak, 3),
                      "status": ops.read_status(dev)}))


if __name__ == "__main__":
    main()
