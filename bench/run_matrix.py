"""Run the headline benchmark at several GPU counts of one node and collect
the JSON lines (the B200 counterpart of the reference's fleet-bench drivers,
experiments/fleet-bench/*.ps1: 1- and 2-stage 8B runs).

    python bench/run_matrix.py --gpus 1,2,4,8 [--steps 32 --warmup 4] [bench.py args...]

N = 1 runs ``python bench.py``; N > 1 runs it under
``torch.distributed.run`` (one rank per GPU, rendezvous on 127.0.0.1), each
under a time limit.  Prints one JSON line per N and a summary table of
tokens/s, ms/step and the speed-up over N = 1 (every number is the bench's
own device-timed max over ranks).
"""
import argparse
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def run_one(n: int, steps: int, warmup: int, extra, port: int, limit: int):
    base = [sys.executable]
    if n > 1:
        base += ["-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
                 "--master-addr", "127.0.0.1", "--master-port", str(port)]
    cmd = ["timeout", "-k", "60", str(limit)] + base + [
        os.path.join(ROOT, "bench.py"), "--gpus", str(n), "--steps", str(steps),
        "--warmup", str(warmup)] + list(extra)
    p = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True)
    for line in reversed(p.stdout.splitlines()):
        line = line.strip()
        if line.startswith("{") and '"metric"' in line:
            return json.loads(line), p.returncode
    return {"n_gpus": n, "error": (p.stderr or p.stdout)[-400:]}, p.returncode


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", default="1,2,4,8")
    ap.add_argument("--steps", type=int, default=32)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--port", type=int, default=29611)
    ap.add_argument("--limit", type=int, default=900, help="seconds per run")
    a, extra = ap.parse_known_args()
    rows = []
    for i, n in enumerate(int(x) for x in a.gpus.split(",")):
        res, rc = run_one(n, a.steps, a.warmup, extra, a.port + i, a.limit)
        print(json.dumps(res), flush=True)
        rows.append(res)
    one = next((r.get("value") for r in rows if r.get("n_gpus") == 1 and "value" in r), None)
    print(f"{'N':>3} {'tokens/s':>12} {'ms/step':>9} {'x N=1':>7}")
    for r in rows:
        if "value" not in r:
            print(f"{r.get('n_gpus', '?'):>3} {'failed':>12}")
            continue
        sp = r["value"] / one if one else float("nan")
        print(f"{r['n_gpus']:>3} {r['value']:>12.1f} {r['ms_per_step']:>9.3f} {sp:>7.2f}")


if __name__ == "__main__":
    main()
