"""bf16 GEMM microbench: our tcgen05 kernel against cuBLAS (torch.matmul) on
the bf16 projections of the sparse-MoE configs, graph-timed.

    python bench/bench_gemm_bf16.py [--m 32] [--shapes qwen3_30b] [--splits 0]

Each shape rotates over enough weight copies that the weights come from HBM
(more than the 126 MB L2 per rotation), a CUDA graph of `reps` launches is
timed with CUDA events after a warm-up replay, and the weight bytes per
launch over the time give the achieved bandwidth (fraction of the measured
HBM copy bandwidth, 6432 GB/s).  One JSON line per shape and implementation.
"""
import argparse
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import torch  # noqa: E402

from cascadia_b200 import ops  # noqa: E402

HBM_GBS = 6432.4
SHAPES = {
    # name: (N, K)
    "qwen3_30b": {"qkv": (5120, 2048), "o": (2048, 4096)},
    "prefill": {"qkv": (5120, 2048), "o": (2048, 4096)},
}


def timed_graph(fn, reps):
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for i in range(reps):
            fn(i)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for i in range(reps):
            fn(i)
    g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    g.replay()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) * 1000 / reps  # us per launch


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--m", type=int, nargs="*", default=[32])
    p.add_argument("--shapes", default="qwen3_30b")
    p.add_argument("--splits", type=int, default=0)
    p.add_argument("--reps", type=int, default=20)
    a = p.parse_args()
    dev = torch.device("cuda")
    for m in a.m:
        for name, (n, k) in SHAPES[a.shapes].items():
            copies = max(2, int(256e6 // (n * k * 2)) + 1)
            ws = [(torch.randn(n, k, device=dev) * 0.05).to(torch.bfloat16) for _ in range(copies)]
            x = torch.randn(m, k, device=dev).to(torch.bfloat16)
            outs = [torch.empty(m, n, dtype=torch.bfloat16, device=dev) for _ in range(2)]
            ours = lambda i: ops.bf16_gemm(x, ws[i % copies], out=outs[i % 2], splits=a.splits)
            lib = lambda i: torch.matmul(x, ws[i % copies].t(), out=outs[i % 2])
            plan = ops.ext().bf16_gemm_plan(m, n, k, a.splits)
            for impl, fn in (("tcgen05", ours), ("cublas", lib)):
                us = timed_graph(fn, a.reps)
                gbs = (n * k * 2 + m * k * 2 + m * n * 2) / (us * 1e-6) / 1e9
                tf = 2 * m * n * k / (us * 1e-6) / 1e12
                print(json.dumps({"shape": name, "m": m, "n": n, "k": k, "impl": impl,
                                  "us": round(us, 2), "GB_s": round(gbs, 1),
                                  "frac_hbm_of_measured": round(gbs / HBM_GBS, 3),
                                  "tflops": round(tf, 1),
                                  "plan": plan[:4] if impl == "tcgen05" else None}))
            assert ops.read_status(dev) == 0


if __name__ == "__main__":
    main()
