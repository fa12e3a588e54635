"""Device topology: nodes (GPUs / hosts) and measured links.

Same data model and JSON as the reference's topology graph
(crates/cascadia-topology/src/lib.rs:25-105: ``NodeInfo``, ``EdgeMetrics``,
directed edges keyed by (src, dst), stale-node expiry) and its
``/api/topology`` response (crates/cascadia-dashboard/src/lib.rs:96-125).
On a B200 box the nodes are the GPUs and the edges are NVLink paths,
measured by :func:`probe_gpus` (peer copy bandwidth and small-copy latency
between every pair of GPUs with peer access).  Only reads state and copies
buffers; changes no GPU setting.
"""
from __future__ import annotations

import socket
import threading
import time
from dataclasses import asdict, dataclass, field
from typing import Dict, List, Optional, Tuple


def _now() -> float:
    return time.time()


@dataclass
class NodeInfo:
    node_id: str
    host: str
    port: int
    api_port: Optional[int] = None
    namespace: str = "default"
    device: str = "CPU"
    memory_mb: int = 0
    cpu_model: str = ""
    cpu_cores: int = 0
    os: str = ""
    engines: List[str] = field(default_factory=list)
    last_seen: float = field(default_factory=_now)

    def to_json(self) -> dict:
        d = asdict(self)
        if d["api_port"] is None:
            del d["api_port"]
        return d


@dataclass
class EdgeMetrics:
    latency_ms: float = 0.0
    bandwidth_mbps: float = 0.0
    last_measured: float = 0.0


class Topology:
    """Thread-safe directed graph of nodes and measured edges."""

    def __init__(self):
        self._lock = threading.RLock()
        self._nodes: Dict[str, NodeInfo] = {}
        self._edges: Dict[Tuple[str, str], EdgeMetrics] = {}

    def add_node(self, info: NodeInfo):
        with self._lock:
            info.last_seen = _now()
            self._nodes[info.node_id] = info

    def touch(self, node_id: str):
        with self._lock:
            if node_id in self._nodes:
                self._nodes[node_id].last_seen = _now()

    def remove_node(self, node_id: str):
        with self._lock:
            self._nodes.pop(node_id, None)
            for k in [k for k in self._edges if node_id in k]:
                del self._edges[k]

    def measure(self, src: str, dst: str, latency_ms: float, bandwidth_mbps: float):
        with self._lock:
            self._edges[(src, dst)] = EdgeMetrics(latency_ms, bandwidth_mbps, _now())

    def record_latency(self, src: str, dst: str, latency_ms: float):
        with self._lock:
            e = self._edges.setdefault((src, dst), EdgeMetrics())
            e.latency_ms = latency_ms
            e.last_measured = _now()

    def nodes(self) -> List[NodeInfo]:
        with self._lock:
            return list(self._nodes.values())

    def node(self, node_id: str) -> Optional[NodeInfo]:
        with self._lock:
            return self._nodes.get(node_id)

    def edges(self) -> List[Tuple[Tuple[str, str], EdgeMetrics]]:
        with self._lock:
            return list(self._edges.items())

    def edge(self, src: str, dst: str) -> Optional[EdgeMetrics]:
        with self._lock:
            return self._edges.get((src, dst))

    def expire_stale(self, max_age_s: float) -> List[str]:
        """Drop nodes not seen for max_age_s (and their edges)."""
        cutoff = _now() - max_age_s
        with self._lock:
            stale = [n for n, i in self._nodes.items() if i.last_seen < cutoff]
            for n in stale:
                self.remove_node(n)
            return stale

    def to_json(self) -> dict:
        with self._lock:
            return {
                "nodes": [n.to_json() for n in self._nodes.values()],
                "edges": [{"src": s, "dst": d, "latency_ms": m.latency_ms,
                           "bandwidth_mbps": m.bandwidth_mbps,
                           "last_measured": m.last_measured}
                          for (s, d), m in self._edges.items()],
            }


def local_gpu_topology(port: int = 0, api_port: Optional[int] = None,
                       engines: Optional[List[str]] = None, probe: bool = False,
                       probe_mb: int = 256) -> Topology:
    """One node per visible GPU of this host; with ``probe`` every GPU pair
    with peer access gets a measured edge."""
    import torch

    topo = Topology()
    host = socket.gethostname()
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    for i in range(n):
        p = torch.cuda.get_device_properties(i)
        topo.add_node(NodeInfo(node_id=f"gpu{i}", host=host, port=port, api_port=api_port,
                               device=p.name, memory_mb=p.total_memory // 2**20,
                               engines=list(engines or [])))
    if probe and n > 1:
        for (i, j), (lat, bw) in probe_gpus(probe_mb).items():
            topo.measure(f"gpu{i}", f"gpu{j}", lat, bw)
    return topo


def probe_gpus(size_mb: int = 256, reps: int = 5) -> Dict[Tuple[int, int], Tuple[float, float]]:
    """Peer copy bandwidth (MB/s) and 4 KiB copy latency (ms) for every
    ordered GPU pair with peer access, timed with CUDA events on the source
    device's stream (median of ``reps``)."""
    import statistics

    import torch

    n = torch.cuda.device_count()
    out = {}
    for i in range(n):
        for j in range(n):
            if i == j or not torch.cuda.can_device_access_peer(i, j):
                continue
            src = torch.empty(size_mb << 20, dtype=torch.uint8, device=f"cuda:{i}")
            dst = torch.empty(size_mb << 20, dtype=torch.uint8, device=f"cuda:{j}")
            small_s, small_d = src[:4096], dst[:4096]
            with torch.cuda.device(i):
                dst.copy_(src)  # warm-up: peer mapping
                torch.cuda.synchronize(i)
                bws, lats = [], []
                for _ in range(reps):
                    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    a.record()
                    dst.copy_(src, non_blocking=True)
                    b.record()
                    b.synchronize()
                    bws.append(src.numel() / (a.elapsed_time(b) / 1000) / 1e6)
                    a.record()
                    small_d.copy_(small_s, non_blocking=True)
                    b.record()
                    b.synchronize()
                    lats.append(a.elapsed_time(b))
            out[(i, j)] = (statistics.median(lats), statistics.median(bws))
            del src, dst
    return out
