"""Placement: split ranking with measured inputs, launch command, and the
restart supervisor (fake processes, no GPU)."""
import json

import pytest

from cascadia_b200.utils import placement as pl


def test_measured_bandwidth_from_peaks_file(tmp_path):
    f = tmp_path / "peaks.json"
    f.write_text(json.dumps({"hbm_gbs": 5000.0}))
    assert pl.measured_hbm_gbs(str(f)) == 5000.0
    assert pl.measured_hbm_gbs(str(tmp_path / "missing.json")) == pl.HBM_GBS


def test_ranking_uses_measured_layer_cost():
    a = pl.choose_parallelism("llama-3.1-8b", 8, 64, 1024, hbm_gbs=6400.0)
    assert a["best"] is not None and a["inputs"]["hbm_gbs"] == 6400.0
    # A slower measured layer makes every candidate slower by the same
    # layer work; collectives are unchanged, so TP=8 gains relative to TP=1.
    b = pl.choose_parallelism("llama-3.1-8b", 8, 64, 1024, layer_us=150.0)
    by = {(c["pp"], c["tp"]): c["decode_step_us"] for c in b["candidates"]}
    assert by[(1, 8)] < by[(8, 1)] * 1.5
    assert b["inputs"]["layer_us"] == 150.0
    # Memory: a 70 GB-per-GPU cap rejects splits that do not fit.
    c = pl.choose_parallelism("qwen3-30b-a3b", 8, 32, 2048, gpu_mem_gb=10.0)
    assert all(x["mem_gb_per_gpu"] <= 10.0 for x in c["candidates"])


def test_launch_command_and_supervisor():
    cmd = pl.launch_command("llama-3.1-8b", {"pp": 2, "tp": 4, "ep": 1}, api="127.0.0.1:9000")
    assert "--nproc-per-node=8" in cmd and cmd[cmd.index("--tp") + 1] == "4"
    assert cmd[cmd.index("--pp") + 1] == "2" and "127.0.0.1" in cmd
    with pytest.raises(ValueError):
        pl.launch_command("qwen3-30b-a3b", {"pp": 1, "tp": 1, "ep": 8})

    codes = iter([1, 1, 0])
    started = []

    class P:
        def __init__(self, c):
            started.append(c)
            self.code = next(codes)

        def wait(self):
            return self.code

    sleeps = []
    assert pl.supervise(["x"], max_restarts=3, popen=P, sleep=sleeps.append) == 0
    assert len(started) == 3 and sleeps == [2.0, 4.0]
    codes2 = iter([7, 7, 7])

    class Q(P):
        def __init__(self, c):
            self.code = next(codes2)

    assert pl.supervise(["x"], max_restarts=2, popen=Q, sleep=lambda s: None) == 7


def test_cli_place_prints_launch_line(capsys):
    from cascadia_b200.cli import main

    main(["place", "--model", "llama-3.1-8b", "--gpus", "4", "--batch", "64"])
    out = json.loads(capsys.readouterr().out)
    assert out["best"] and "torch.distributed.run" in out["launch"]
