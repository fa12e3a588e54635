"""Topology graph (reference data model) and its API / dashboard routes."""
import time

import pytest
import torch
from fastapi.testclient import TestClient

from cascadia_b200.topology import NodeInfo, Topology


def test_topology_graph_and_expiry():
    t = Topology()
    t.add_node(NodeInfo("a", "h1", 9000, api_port=8000, device="B200"))
    t.add_node(NodeInfo("b", "h1", 9001))
    t.measure("a", "b", 0.01, 770000.0)
    t.record_latency("b", "a", 0.02)
    j = t.to_json()
    assert {n["node_id"] for n in j["nodes"]} == {"a", "b"}
    assert "api_port" not in [n for n in j["nodes"] if n["node_id"] == "b"][0]
    e = {(x["src"], x["dst"]): x for x in j["edges"]}
    assert e[("a", "b")]["bandwidth_mbps"] == 770000.0 and e[("b", "a")]["latency_ms"] == 0.02
    t.node("b").last_seen = time.time() - 100
    assert t.expire_stale(10) == ["b"]
    assert t.edges() == []


def test_dashboard_and_topology_routes():
    from cascadia_b200.api.server import make_app
    from cascadia_b200.engine.mock import MockBuilder
    from cascadia_b200.runtime.runner import Runner
    from cascadia_b200.types import PeerLayout, ShardSpec

    r = Runner(MockBuilder(), model_id="m", device="cpu")
    r.start(PeerLayout(), ShardSpec("m", 0, 1, 1))
    t = Topology()
    t.add_node(NodeInfo("gpu0", "h", 0, device="B200"))
    with TestClient(make_app(r, topology=t)) as c:
        assert c.get("/api/topology").json()["nodes"][0]["device"] == "B200"
        assert "/api/topology" in c.get("/").text
    r.close()


@pytest.mark.gpu
def test_local_gpu_topology_probe():
    from cascadia_b200.topology import local_gpu_topology

    t = local_gpu_topology(probe=True, probe_mb=64)
    n = torch.cuda.device_count()
    assert len(t.nodes()) == n
    if n > 1:
        assert len(t.edges()) == n * (n - 1)
        assert all(m.bandwidth_mbps > 0 for _, m in t.edges())
