"""W4A16 GEMM microbenchmark on the Llama-3.1-8B layer shapes.

    python bench/bench_gemm.py [--m 64] [--shapes qkv,o,gate_up,down,lm_head] [--reps 20]

Times each GEMM with CUDA events around a CUDA graph of `reps` launches
(after warm-up; weight copies rotate so each launch reads its weights from
HBM, not L2; the graph removes the host launch cost, as in decode) and reports
achieved HBM bandwidth of the weight stream against MEASURED_PEAKS.json.
``--reps 1 --shapes gate_up`` gives a single launch for an ncu capture.
"""
import argparse
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import torch  # noqa: E402

from cascadia_b200 import ops  # noqa: E402
from cascadia_b200.quant import Int4Weight, blob_bytes  # noqa: E402

SHAPES = {  # name: (N, K, epilogue)
    "qkv": (6144, 4096, ops.EPI_STORE),
    "o": (4096, 4096, ops.EPI_RESID),
    "gate_up": (28672, 4096, ops.EPI_SILU),
    "down": (4096, 14336, ops.EPI_RESID),
    "lm_head": (128256, 4096, ops.EPI_STORE),
}


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--m", type=int, default=64)
    p.add_argument("--shapes", default="qkv,o,gate_up,down,lm_head")
    p.add_argument("--reps", type=int, default=20)
    p.add_argument("--copies", type=int, default=4, help="weight copies rotated per shape")
    p.add_argument("--splits", type=int, default=0,
                   help="0 auto; > 0 split-K kernel with that split; "
                        "-2 small-M kernel")
    p.add_argument("--graph", type=int, default=1, help="time a CUDA graph of the reps launches")
    p.add_argument("--tp", type=int, default=1,
                   help="shapes of one tensor-parallel rank (N or K divided by tp)")
    p.add_argument("--sweep-splits", default="",
                   help="comma-separated split-K factors to time per shape (best reported)")
    p.add_argument("--trace", action="store_true",
                   help="tcgen05 path: print per-CTA phase times of one launch")
    a = p.parse_args()
    dev = torch.device("cuda", 0)
    peak = 6432.4
    pk = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                      "MEASURED_PEAKS.json")
    if os.path.exists(pk):
        peak = json.load(open(pk)).get("hbm_gbs", peak)
    res = {}
    for name in a.shapes.split(","):
        n, k, epi = SHAPES[name]
        if a.tp > 1:
            # Column-parallel: rows split (lm_head padded to 128-row tiles);
            # row-parallel (o, down): K split.
            if name in ("o", "down"):
                k //= a.tp
            elif name == "lm_head":
                n = -(-n // (a.tp * 128)) * 128
            else:
                n //= a.tp
        if a.sweep_splits:
            sweep = [int(x) for x in a.sweep_splits.split(",")]
            g = torch.Generator(device=dev).manual_seed(0)
            blobs = [Int4Weight.random(n, k, generator=g, device=dev).blob(epi == ops.EPI_SILU)
                     for _ in range(a.copies)]
            x = torch.randn(a.m, k, device=dev).to(torch.bfloat16)
            resid = torch.randn(a.m, n, device=dev).to(torch.bfloat16)
            outs = torch.empty(a.m, n, dtype=torch.bfloat16, device=dev)
            times = {}
            for sp in sweep:
                if sp > k // 128:
                    continue

                def run_s(i, sp=sp):
                    kw = dict(residual=resid, out=outs) if epi == ops.EPI_RESID else {}
                    return ops.w4a16_gemm(x, blobs[i % a.copies], n, 128, epi, splits=sp, **kw)
                for i in range(3):
                    run_s(i)
                torch.cuda.synchronize()
                gr = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gr):
                    for i in range(a.reps):
                        run_s(i)
                gr.replay()
                torch.cuda.synchronize()
                ts = []
                for _ in range(3):
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record()
                    gr.replay()
                    e1.record()
                    torch.cuda.synchronize()
                    ts.append(e0.elapsed_time(e1) * 1000 / a.reps)
                times[sp] = round(min(ts), 2)
                del gr
            auto = ops.w4a16_plan(a.m, n, k, 0)
            best = min(times, key=times.get)
            print(name, json.dumps({"n": n, "k": k, "m": a.m, "us_by_splits": times,
                                    "best_splits": best, "auto_plan": auto}), flush=True)
            continue
        g = torch.Generator(device=dev).manual_seed(0)
        copies = a.copies if a.reps > 1 else 1
        blobs = [Int4Weight.random(n, k, generator=g, device=dev).blob(epi == ops.EPI_SILU)
                 for _ in range(copies)]
        x = torch.randn(a.m, k, device=dev).to(torch.bfloat16)
        resid = torch.randn(a.m, n, device=dev).to(torch.bfloat16)
        outs = torch.empty(a.m, n, dtype=torch.bfloat16, device=dev)

        def run(i):
            kw = {}
            if epi == ops.EPI_RESID:
                kw = dict(residual=resid, out=outs)
            return ops.w4a16_gemm(x, blobs[i % copies], n, 128, epi, splits=a.splits, **kw)

        for i in range(min(3, a.reps)):
            run(i)
        torch.cuda.synchronize()
        if a.graph and a.reps > 1:
            # Launch-overhead-free timing: the reps launches captured in one
            # CUDA graph, replayed; per-launch time = replay time / reps.
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr):
                for i in range(a.reps):
                    run(i)
            gr.replay()
            torch.cuda.synchronize()
            ts = []
            for _ in range(5):
                s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s0.record()
                gr.replay()
                s1.record()
                torch.cuda.synchronize()
                ts.append(s0.elapsed_time(s1) * 1000 / a.reps)
            ts.sort()
            del gr
        else:
            ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                  for _ in range(a.reps)]
            for i in range(a.reps):
                ev[i][0].record()
                run(i)
                ev[i][1].record()
            torch.cuda.synchronize()
            ts = sorted(s.elapsed_time(e) * 1000 for s, e in ev)
        med = ts[len(ts) // 2]
        nbytes = blob_bytes(n, k, 128) + a.m * k * 2 + a.m * n * 2
        plan = ops.w4a16_plan(a.m, n, k, a.splits)
        res[name] = {"us": round(med, 2), "GBps": round(nbytes / med / 1e3, 1),
                     "frac_of_measured_hbm": round(nbytes / med / 1e3 / peak, 3),
                     "plan": plan,
                     "path": {0: "split-K tcgen05", 2: "small-M"}[plan[0]]}
        print(name, json.dumps(res[name]), flush=True)
        if a.trace and plan[0] == 0:
            buf = torch.zeros(1 << 20, dtype=torch.int64, device=dev)
            ops.ext().w4a16_set_trace(buf)
            run(0)
            torch.cuda.synchronize()
            ops.ext().w4a16_set_trace(None)
            _, mt, sp, _, tt, rt = plan
            n = rt * max(sp, 1) * tt
            names = ["setup", "first_w", "issued", "last_mma", "acc_ready", "partials", "end"]
            width = 8
            tr = buf[:n * width].view(n, width).double().cpu()
            t0 = tr[:, 0].min()
            rel = tr - tr[:, :1]
            print("  CTA start skew us: max", round(float(tr[:, 0].max() - t0) / 1000, 2),
                  "kernel span us", round(float(tr[:, 7].max() - t0) / 1000, 2), flush=True)
            for i, nm in enumerate(names):
                col = rel[:, i + 1] / 1000
                q = torch.quantile(col, torch.tensor([0.1, 0.5, 0.9, 1.0], dtype=col.dtype))
                print(f"    {nm:14s} p10/p50/p90/max us:", [round(float(v), 2) for v in q])
    print("status", ops.read_status(dev))


if __name__ == "__main__":
    main()
