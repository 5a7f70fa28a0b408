"""Devices, fit and spare pools through the real binaries.

Each daemon lists its GPUs with a stand-in for ``nvidia-smi`` (a script that answers the same
query), the coordinator admits or refuses spares by the fit of their device to the rank's, and a
pool launches spares on free devices of its class. The last test runs an engine whose only
spare is a pool's spare for any rank: it takes the killed rank and the streams stay
token-identical.
"""

import os
import stat
import subprocess
import sys

import pytest
import torch

from everserve_b200.contract.daemon import DaemonConnection
from everserve_b200.proto import signals as sp
from everserve_b200.serving.cluster import ControlPlane, binary

from test_control_cpu import _P, _wait


def _fake_smi(path, rows):
    """A program answering `--query-gpu=index,uuid,name,memory.total --format=csv,noheader,nounits`."""
    with open(path, "w") as f:
        f.write("#!/bin/sh\ncat <<'EOF'\n" + "".join(f"{i}, GPU-{path[-6:]}-{i}, {name}, {mib}\n"
                                                  for i, (name, mib) in enumerate(rows)) + "EOF\n")
    os.chmod(path, os.stat(path).st_mode | stat.S_IEXEC)
    return str(path)


class _Dev(_P):
    def __init__(self, rank, device):
        super().__init__(rank)
        self.device = device

    def identity(self):
        return self.rank, self.device


def test_coordinator_unit_checks():
    r = subprocess.run([binary("everserve-coord-tests")], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stderr
    assert "all checks passed" in r.stdout


def test_device_fit_refuses_a_slower_spare_and_pools_place_by_class(tmp_path):
    b200 = _fake_smi(str(tmp_path / "smi-n0"), [("NVIDIA B200", 183359)] * 2)
    h100 = _fake_smi(str(tmp_path / "smi-n1"), [("NVIDIA H100 80GB HBM3", 81559)] * 2)
    marker = tmp_path / "launched.txt"
    with ControlPlane(str(tmp_path / "cp"), engines=[{"name": "e0", "tensorParallel": 2}], extra_nodes=["n1"],
                      node_extra={"n0": ["--devices-from", b200, "--domain", "rackA"],
                                  "n1": ["--devices-from", h100]}) as cp:
        nodes = {n["metadata"]["name"]: n["status"] for n in cp.get("/v1/nodes")["items"]}
        assert [d["class"] for d in nodes["n0"]["devices"]] == ["NVIDIA B200"] * 2
        assert nodes["n0"]["devices"][0]["memoryBytes"] == 183359 << 20
        assert nodes["n0"]["domain"] == "rackA" and nodes["n1"]["domain"] == "n1"
        w0 = DaemonConnection(cp.daemon_sockets["n0"], "e0", _Dev(0, 0), node="n0")
        w1 = DaemonConnection(cp.daemon_sockets["n0"], "e0", _Dev(1, 1), node="n0")
        assert _wait(lambda: len(cp.engine_view("e0")["status"]["workers"]) == 2)
        # a spare for rank 1 on an H100: 58 % slower than the B200 it would replace, refused
        s1 = DaemonConnection(cp.daemon_sockets["n1"], "e0", _Dev(1, 0), node="n1", role=sp.ROLE_SPARE)
        assert _wait(lambda: cp.engine_view("e0")["status"]["refusedSpares"])
        st = cp.engine_view("e0")["status"]
        assert st["spares"] == []
        why = st["refusedSpares"][0]["why"]
        assert "H100" in why and "B200" in why and "mismatched" in why, why
        assert any("refused" in ev["text"] for ev in cp.get("/v1/engines/e0/events")["events"])

        # pools: an unknown engine and a stale generation are refused
        code, body = cp.request("PUT", "/v1/pools/p0", {"engines": ["nope"], "wants": 1})
        assert code == 400 and "nope" in body["error"]
        code, body = cp.request("PUT", "/v1/pools/p0", {"engines": ["e0"], "wants": 1, "deviceClass": "B200",
                                                         "command": ["sleep", "30"]})
        assert code == 200 and body["metadata"]["generation"] == 1
        # every B200 holds a worker: nothing to launch, the pool is short
        assert body["status"]["short"] == 1 and body["status"]["warming"] == 0
        code, body = cp.request("PUT", "/v1/pools/p0?generation=7", {"engines": ["e0"], "wants": 1})
        assert code == 409
        # an H100 pool launches on n1's free device (device 0 holds the refused spare)
        cmd = ["sh", "-c", f"echo {{pool}} {{node}} {{device}} {{engines}} > {marker}; sleep 30"]
        code, body = cp.request("PUT", "/v1/pools/p1", {"engines": ["e0"], "wants": 1, "deviceClass": "H100",
                                                         "command": cmd})
        assert code == 200 and body["status"]["warming"] == 1
        assert _wait(lambda: marker.exists() and marker.read_text().strip(), timeout=15)
        assert marker.read_text().split() == ["p1", "n1", "1", "e0"]
        assert {p["metadata"]["name"] for p in cp.get("/v1/pools")["items"]} == {"p0", "p1"}
        code, _ = cp.request("DELETE", "/v1/pools/p0")
        assert code == 200
        assert {p["metadata"]["name"] for p in cp.get("/v1/pools")["items"]} == {"p1"}
        # the pool's spec survives in the spec store
        assert os.path.exists(os.path.join(cp.dir, "spec", "pools", "p1.json"))
        # the operator CLI writes and reads pools too
        spec = tmp_path / "p2.json"
        spec.write_text('{"engines": ["e0"], "wants": 0, "reason": "headroom"}')
        ctl = [binary("everserve-ctl"), "--api", cp.api]
        assert subprocess.run(ctl + ["pool", "apply", "p2", str(spec)], capture_output=True).returncode == 0
        r = subprocess.run(ctl + ["pool", "apply", "p2", str(spec), "--generation", "5"], capture_output=True)
        assert r.returncode != 0  # generation 1 is held
        out = subprocess.run(ctl + ["get", "pool", "p2"], capture_output=True, text=True).stdout
        assert '"reason":"headroom"' in out and '"generation":1' in out
        for c in (w0, w1, s1):
            c.close()


def test_mismatched_spare_admitted_within_the_policys_degrade(tmp_path):
    b200 = _fake_smi(str(tmp_path / "smi-n0"), [("NVIDIA B200", 183359)] * 2)
    h200 = _fake_smi(str(tmp_path / "smi-n1"), [("NVIDIA H200", 143771)])
    with ControlPlane(str(tmp_path / "cp"), engines=[{"name": "e0", "tensorParallel": 2}], extra_nodes=["n1"],
                      node_extra={"n0": ["--devices-from", b200], "n1": ["--devices-from", h200]},
                      policy_extra={"spares": {"allowMismatched": True, "maxDegradePercent": 50}}) as cp:
        w0 = DaemonConnection(cp.daemon_sockets["n0"], "e0", _Dev(0, 0), node="n0")
        w1 = DaemonConnection(cp.daemon_sockets["n0"], "e0", _Dev(1, 1), node="n0")
        assert _wait(lambda: len(cp.engine_view("e0")["status"]["workers"]) == 2)
        s = DaemonConnection(cp.daemon_sockets["n1"], "e0", _Dev(1, 0), node="n1", role=sp.ROLE_SPARE)
        # an H200 in place of a B200 runs at 0.6 of its speed: 40 % slower, within 50 %
        assert _wait(lambda: cp.engine_view("e0")["status"]["spares"])
        assert cp.engine_view("e0")["status"]["refusedSpares"] == []
        # a cordoned node's spare is refused, and stands again when uncordoned
        cp.request("PUT", "/v1/nodes/n1/cordon")
        assert _wait(lambda: not cp.engine_view("e0")["status"]["spares"])
        assert "cordoned" in cp.engine_view("e0")["status"]["refusedSpares"][0]["why"]
        cp.request("PUT", "/v1/nodes/n1/uncordon")
        assert _wait(lambda: cp.engine_view("e0")["status"]["spares"])
        for c in (w0, w1, s):
            c.close()


@pytest.mark.slow
def test_pool_spare_for_any_rank_takes_over_token_identical(tmp_path):
    """A pool of one spare for e0 on the node's free device: the daemon launches it, it fetches
    the start-up record, stands for any rank holding no shard, and when rank 1 is killed it
    builds rank 1, restores its committed KV and takes it. The streams stay token-identical."""
    from everserve_b200.engine.config import EngineConfig
    from everserve_b200.engine.engine import Engine
    from everserve_b200.serving.executor import MultiprocExecutor, failover

    from test_failover_cpu import KILL_AT, MODEL, PROMPT, STREAMS, TOKENS, _prompts, _run

    base, _, _, _ = _run(tmp_path / "nofault", spares=())
    cfg = EngineConfig(model=MODEL, device="cpu", dtype=torch.float32, num_blocks=128, max_batch=STREAMS,
                       max_model_len=PROMPT + TOKENS + 16, pipeline_parallel=2, use_cuda_graphs=False)
    smi = _fake_smi(str(tmp_path / "smi"), [("NVIDIA B200", 183359)] * 3)  # ranks 0 and 1 hold devices 0, 1
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    with ControlPlane(str(tmp_path / "pool"), engines=[{"name": "e0", "pipelineParallel": 2}],
                      node_args=["--devices-from", smi]) as cp:
        ex = MultiprocExecutor(cfg, engine="e0", daemon=cp.daemon_socket, store=cp.store_socket, spares=(),
                               node="n0", log_dir=str(tmp_path / "pool" / "logs"), threads=2)
        try:
            code, _ = cp.request("PUT", "/v1/pools/p0", {
                "engines": ["e0"], "wants": 1, "deviceClass": "B200",
                "command": [sys.executable, "-m", "everserve_b200.serving.spare"],
                "env": {"PYTHONPATH": root}})
            assert code == 200
            cp.wait_spares("e0", 1, timeout_s=300)
            spare = cp.engine_view("e0")["status"]["spares"][0]
            assert spare["forRank"] == -1 and spare["pool"] == "p0" and spare["device"] == 2
            eng = Engine(cfg, executor=ex)
            eng.wrap_step(failover(ex, eng))
            ex.kill_at_decode_step = (KILL_AT, 1)
            out = eng.generate(_prompts(), max_tokens=TOKENS)
            assert len(ex.changes) == 1 and out == base
            workers = {w["rank"]: w for w in cp.engine_view("e0")["status"]["workers"]}
            assert workers[1]["device"] == 2  # the pool's device holds rank 1 now
            # its spare is spent; the lost rank's device is free again, and the pool launches there
            assert _wait(lambda: cp.get("/v1/pools/p0")["status"]["short"] == 0, timeout=30)
        finally:
            ex.shutdown()


def test_node_reclaimable_and_expected_pause(tmp_path):
    with ControlPlane(str(tmp_path / "cp"), engines=[{"name": "e0", "tensorParallel": 2}], extra_nodes=["n1"]) as cp:
        w0 = DaemonConnection(cp.daemon_sockets["n0"], "e0", _Dev(0, 0), node="n0")
        w1 = DaemonConnection(cp.daemon_sockets["n0"], "e0", _Dev(1, 1), node="n0")
        assert _wait(lambda: len(cp.engine_view("e0")["status"]["workers"]) == 2)
        nodes = {n["metadata"]["name"]: n["status"] for n in cp.get("/v1/nodes")["items"]}
        assert nodes["n0"]["reclaimable"] is False and "rank 0" in nodes["n0"]["reclaimBlocker"]
        assert nodes["n1"]["reclaimable"] is True  # holds nothing
        assert cp.engine_view("e0")["status"]["expectedPauseMs"] is None
        # one spare for any rank on n1: n0 holds two ranks, so it is still not reclaimable
        s1 = DaemonConnection(cp.daemon_sockets["n1"], "e0", _Dev(0, 0), node="n1", role=sp.ROLE_SPARE, any_rank=True)
        assert _wait(lambda: cp.engine_view("e0")["status"]["spares"])
        nodes = {n["metadata"]["name"]: n["status"] for n in cp.get("/v1/nodes")["items"]}
        assert nodes["n0"]["reclaimable"] is False and "rank 1" in nodes["n0"]["reclaimBlocker"]
        s2 = DaemonConnection(cp.daemon_sockets["n1"], "e0", _Dev(1, 1), node="n1", role=sp.ROLE_SPARE)
        assert _wait(lambda: {n["metadata"]["name"]: n["status"] for n in cp.get("/v1/nodes")["items"]}["n0"]["reclaimable"])
        # a change gives the engine an observed pause (rank 1's connection ends: a departure; a
        # reported loss of a rank whose process still runs would have its daemon fence it, and
        # here that process is this test's)
        w1.close(sp.STOP_CAUSE_LOST)
        assert _wait(lambda: cp.engine_view("e0")["status"]["expectedPauseMs"] is not None, timeout=15)
        for c in (w0, s1, s2):
            c.close()
