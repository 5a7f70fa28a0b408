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
    t0 = time.monotonic()
    while time.monotonic() - t0 < timeout:
        if pred():
            return True
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
