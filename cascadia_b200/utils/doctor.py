"""Environment checks (`cascadia_b200 doctor`).

The reference's doctor checks Rust / C++ / OpenVINO devices
(crates/cascadia-cli/src/doctor.rs:93-282); on a B200 box the questions are:
is the CUDA driver there, are the GPUs sm_100, is our sm_100a extension built
and loadable, which NCCL is linked, and can every GPU reach every peer over
NVLink (P2P access matrix).  Only reads state; changes no GPU setting.
"""
from __future__ import annotations

import shutil
import subprocess


def run_doctor() -> dict:
    import torch

    rep = {"torch": torch.__version__, "cuda_runtime": torch.version.cuda, "checks": []}

    def check(name, ok, detail=""):
        rep["checks"].append({"check": name, "ok": bool(ok), "detail": str(detail)})
        return ok

    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    check("cuda_available", n > 0, f"{n} device(s)")
    caps = []
    for i in range(n):
        p = torch.cuda.get_device_properties(i)
        caps.append({"index": i, "name": p.name, "cc": f"{p.major}.{p.minor}",
                     "sms": p.multi_processor_count, "mem_gb": round(p.total_memory / 2**30, 1)})
    rep["devices"] = caps
    check("sm_100", all(c["cc"] == "10.0" for c in caps) and caps, caps)
    try:
        from .. import _C  # noqa: F401

        check("extension_sm100a", True, "cascadia_b200._C loaded")
    except Exception as e:  # noqa: BLE001
        check("extension_sm100a", False, e)
    try:
        from .. import _runtime  # noqa: F401

        check("native_runtime", True, "cascadia_b200._runtime loaded")
    except Exception as e:  # noqa: BLE001
        check("native_runtime", False, e)
    try:
        v = torch.cuda.nccl.version()
        check("nccl", True, ".".join(map(str, v)) if isinstance(v, tuple) else v)
    except Exception as e:  # noqa: BLE001
        check("nccl", False, e)
    p2p = [[torch.cuda.can_device_access_peer(i, j) if i != j else True for j in range(n)]
           for i in range(n)]
    rep["p2p_matrix"] = p2p
    check("p2p_all_pairs", all(all(r) for r in p2p), "")
    if shutil.which("nvidia-smi"):
        try:
            topo = subprocess.run(["nvidia-smi", "topo", "-m"], capture_output=True, text=True,
                                  timeout=20).stdout
            rep["topology"] = topo
        except Exception as e:  # noqa: BLE001
            rep["topology"] = str(e)
    rep["ok"] = all(c["ok"] for c in rep["checks"])
    return rep
