"""Control-plane behaviours through the real binaries and the Python contract: undecided processes
get roles, stack dumps reach the operator, stale loss reports are fenced."""

import os
import threading
import time

from everserve_b200.contract.daemon import DaemonConnection, UndecidedConnection
from everserve_b200.proto import signals as sp
from everserve_b200.serving.cluster import ControlPlane


class _P:
    def __init__(self, rank):
        self.rank = rank
        self.changes = []

    def identity(self):
        return self.rank, 0

    def on_change(self, ch):
        self.changes.append(ch)

    def on_notice(self, *a):
        pass

    def on_abandoned(self, *a):
        pass

    def on_committed(self, c):
        pass

    def on_join(self, j):
        pass

    def on_displaced(self, *a):
        pass


def _wait(pred, timeout=10.0):
    """Poll `pred` until it holds; a view the coordinator has not made yet (404) counts as not yet."""
    t0 = time.monotonic()
    while time.monotonic() - t0 < timeout:
        try:
            if pred():
                return True
        except (ValueError, KeyError):
            pass
        time.sleep(0.02)
    return False


def test_undecided_gets_worker_then_spare(tmp_path):
    with ControlPlane(str(tmp_path), engines=[{"name": "e0", "tensorParallel": 2}]) as cp:
        w0 = DaemonConnection(cp.daemon_socket, "e0", _P(0), node="n0")
        assert _wait(lambda: any(w["rank"] == 0 for w in cp.engine_view("e0")["status"]["workers"]))
        u1 = UndecidedConnection(cp.daemon_socket, "e0", rank=1, node="n0")
        assert u1.assigned(timeout_s=10).role == sp.ROLE_WORKER  # rank 1 is free: a worker
        u0 = UndecidedConnection(cp.daemon_socket, "e0", rank=0, node="n0")
        assert u0.assigned(timeout_s=10).role == sp.ROLE_SPARE  # rank 0 is held: a spare
        for c in (w0, u1, u0):
            c.close()


def test_stack_dump_reaches_the_operator(tmp_path):
    with ControlPlane(str(tmp_path), engines=[{"name": "e0"}]) as cp:
        conn = DaemonConnection(cp.daemon_socket, "e0", _P(0), node="n0")
        assert _wait(lambda: cp.engine_view("e0")["status"]["workers"])
        import http.client

        host, port = cp.api.rsplit(":", 1)
        c = http.client.HTTPConnection(host, int(port), timeout=5)
        c.request("POST", "/v1/engines/e0/stacks")
        rid = __import__("json").loads(c.getresponse().read())["requested"]
        assert _wait(lambda: cp.get(f"/v1/stacks/{rid}")["processes"])
        text = cp.get(f"/v1/stacks/{rid}")["processes"][0]["stacks"]
        assert "thread" in text and "daemon-e0-0" in text  # every Python thread's stack, named
        conn.close()


def test_stale_epoch_loss_report_is_fenced(tmp_path):
    """After two changes (epoch 2), a loss report stamped with epoch 1 is from the engine's past
    and is dropped (counted, no change)."""
    import http.client

    with ControlPlane(str(tmp_path), engines=[{"name": "e0", "tensorParallel": 2}]) as cp:
        p0, p1, pa, pb = _P(0), _P(1), _P(1), _P(1)
        c0 = DaemonConnection(cp.daemon_socket, "e0", p0, node="n0")
        c1 = DaemonConnection(cp.daemon_socket, "e0", p1, node="n0")
        ca = DaemonConnection(cp.daemon_socket, "e0", pa, role=sp.ROLE_SPARE, node="n0")
        assert _wait(lambda: len(cp.engine_view("e0")["status"]["workers"]) == 2
                     and cp.engine_view("e0")["status"]["spares"])
        c1.close(cause=sp.STOP_CAUSE_LOST)  # rank 1 goes; spare A takes it: epoch 1
        assert _wait(lambda: cp.engine_view("e0")["status"]["epoch"] == 1)
        assert pa.changes and pa.changes[0].take[0].rank == 1
        cb = DaemonConnection(cp.daemon_socket, "e0", pb, role=sp.ROLE_SPARE, node="n0")
        assert _wait(lambda: cp.engine_view("e0")["status"]["spares"])
        ca.close(cause=sp.STOP_CAUSE_LOST)  # A (now rank 1) goes; spare B takes it: epoch 2
        assert _wait(lambda: cp.engine_view("e0")["status"]["epoch"] == 2)
        c0.report_lost([0], "stale", epoch=1)
        time.sleep(0.5)
        st = cp.engine_view("e0")["status"]
        assert st["epoch"] == 2 and not st["changing"] and not st["down"]
        host, port = cp.api.rsplit(":", 1)
        c = http.client.HTTPConnection(host, int(port), timeout=5)
        c.request("GET", "/metrics")
        text = c.getresponse().read().decode()
        assert any(line.startswith("everserve_fenced_total") and not line.endswith(" 0")
                   for line in text.splitlines())
        for conn in (c0, cb):
            conn.close()


def test_fleet_harness_commits_every_loss_at_scale():
    """The control-plane scale harness against the real coordinator: 72 simulated nodes (64 TP8
    engines, 8 spare nodes); every loss is replaced and committed within the coordinator's
    stamps."""
    import asyncio

    from everserve_b200.perf.fleet import run_fleet
    from everserve_b200.serving.cluster import binary

    r = asyncio.run(run_fleet(binary("everserve-coord"), 72, 8, 8))
    assert r["losses"] == 8 and r["engines"] == 64
    assert 0 < r["report_to_commit_ms"]["max"] < 1000


def test_daemon_fences_a_displaced_worker(tmp_path):
    """A worker whose rank the coordinator gave to a spare while the worker still runs (hung, or
    cut off) is stopped by its node's daemon after the commit."""
    import subprocess
    import sys

    from everserve_b200.proto import signals as sp2

    code = (
        "import time, sys\n"
        "from everserve_b200.contract.daemon import DaemonConnection\n"
        "class P:\n"
        "    def identity(self): return 1, 1\n"
        "    def on_change(self, ch): return None\n"
        "    def on_notice(self, *a): pass\n"
        "    def on_abandoned(self, *a): pass\n"
        "    def on_committed(self, c): pass\n"
        "    def on_join(self, j): pass\n"
        "    def on_displaced(self, *a): pass\n"
        "c = DaemonConnection({cp_sock!r}, 'e0', P(), node='n0')\n"
        "print('registered', flush=True)\n"
        "time.sleep(120)\n"
    )
    with ControlPlane(str(tmp_path), engines=[{"name": "e0", "tensorParallel": 2}], extra_nodes=["n1"]) as cp:
        w0 = DaemonConnection(cp.daemon_sockets["n0"], "e0", _P(0), node="n0")
        hung = subprocess.Popen([sys.executable, "-c", code.replace("{cp_sock!r}", repr(cp.daemon_sockets["n0"]))],
                                stdout=subprocess.PIPE, text=True,
                                env=dict(os.environ, PYTHONPATH=os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
        assert hung.stdout.readline().strip() == "registered"
        spare = DaemonConnection(cp.daemon_sockets["n1"], "e0", _P(1), node="n1", role=sp2.ROLE_SPARE)
        assert _wait(lambda: len(cp.engine_view("e0")["status"]["workers"]) == 2 and
                     cp.engine_view("e0")["status"]["spares"])
        w0.report_lost([1], "rank 1 is hung", reason=sp2.REASON_FAULT)
        assert _wait(lambda: cp.engine_view("e0")["status"]["epoch"] == 1, timeout=15)
        assert hung.wait(timeout=15) != 0  # stopped by its daemon
        assert "fencing e0 rank 1" in cp.log("node")
        for c in (w0, spare):
            c.close()


def test_leaked_release_retires_the_rank_by_notice(tmp_path):
    """A worker that reports a leaked release is retired by notice when a spare can take its rank:
    the change names it as departing, so it finishes its step before the spare takes over."""
    from everserve_b200.proto import signals as sp2

    class Rec(_P):
        def on_change(self, ch):
            self.changes.append(ch)
            return None

    with ControlPlane(str(tmp_path), engines=[{"name": "e0", "tensorParallel": 2}], extra_nodes=["n1"]) as cp:
        r0, r1 = Rec(0), Rec(1)
        w0 = DaemonConnection(cp.daemon_sockets["n0"], "e0", r0, node="n0")
        w1 = DaemonConnection(cp.daemon_sockets["n0"], "e0", r1, node="n0")
        spare = DaemonConnection(cp.daemon_sockets["n1"], "e0", Rec(1), node="n1", role=sp2.ROLE_SPARE)
        assert _wait(lambda: len(cp.engine_view("e0")["status"]["workers"]) == 2 and
                     cp.engine_view("e0")["status"]["spares"])
        w1.report_leak("epoch 0 groups", 12.5, 1)
        assert _wait(lambda: cp.engine_view("e0")["status"]["epoch"] == 1, timeout=15)
        assert r1.changes and list(r1.changes[-1].departing) == [1]
        assert any("leaked a release" in e["text"] for e in cp.get("/v1/engines/e0/events")["events"])
        for c in (w0, w1, spare):
            c.close()
