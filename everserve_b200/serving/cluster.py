"""A one-node control plane in a directory: coordinator, node daemon and KV store.

    with ControlPlane(workdir, engines=[{"name": "e0", "pipelineParallel": 2}]) as cp:
        ... cp.daemon_socket, cp.store_socket, cp.api ...

It starts the C++ binaries (``cpp/bin``; built with ``make -C cpp`` when missing) with their
sockets, spec store, lease and logs under ``workdir``, waits for them to listen, and stops them
on exit. The policy file it writes is ``everserve.policy.v1.Policy`` in proto3 JSON.

This is the bare-metal layout of the reference's deploy/baremetal units (one coordinator per
cluster, one daemon and one store per node), for tests, benchmarks and single-node serving.
"""

from __future__ import annotations

import json
import os
import socket
import subprocess
import time

_ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
BIN = os.path.join(_ROOT, "cpp", "bin")


def binary(name: str) -> str:
    path = os.path.join(BIN, name)
    if not os.path.exists(path):
        subprocess.run(["make", "-C", os.path.join(_ROOT, "cpp"), f"-j{os.cpu_count() or 4}"], check=True,
                       stdout=subprocess.DEVNULL)
    return path


_handed: set[int] = set()


def free_port() -> int:
    """A loopback port no one listens on, never the same one twice in this process.

    Ports come from below the kernel's ephemeral range, so a port handed out now and bound later
    (a standby coordinator binds its API only when it takes the lease) is not given meanwhile to
    some other socket's implicit bind."""
    import random

    lo = 20000
    try:
        with open("/proc/sys/net/ipv4/ip_local_port_range") as f:
            eph = int(f.read().split()[0])
    except (OSError, ValueError):
        eph = 32768
    hi = max(lo + 1000, eph - 1)
    rng = random.Random()
    while True:
        port = rng.randrange(lo, hi)
        if port in _handed:
            continue
        s = socket.socket()
        try:
            s.bind(("127.0.0.1", port))
        except OSError:
            continue
        finally:
            s.close()
        _handed.add(port)
        return port


def wait_listening(addr: str, timeout_s: float = 15.0) -> None:
    deadline = time.monotonic() + timeout_s
    while time.monotonic() < deadline:
        try:
            if addr.startswith("unix:"):
                s = socket.socket(socket.AF_UNIX)
                s.connect(addr[5:])
            else:
                host, _, port = addr.rpartition(":")
                s = socket.create_connection((host, int(port)), timeout=0.2)
            s.close()
            return
        except OSError:
            time.sleep(0.02)
    raise TimeoutError(f"{addr} is not listening")


class ControlPlane:
    def __init__(self, workdir: str, engines: list[dict] | None = None, node: str = "n0", extra_nodes=(),
                 outcomes=("OUTCOME_REPLACE",), heartbeat_ms: int = 500, store_slots: int = 1 << 16,
                 store_budget: int = 8 << 30, ack_timeout_ms: int = 120000, cover: bool = True,
                 standby: bool = False, coord_env: dict | None = None, node_args: list[str] | None = None,
                 node_extra: dict | None = None, policy_extra: dict | None = None):
        """`standby`: a second coordinator waits for the lease and takes over when the first
        exits. `coord_env`: extra environment of the first coordinator. `node_args`: extra flags
        of every daemon; `node_extra`: of one daemon, by node. `policy_extra`: more policy fields
        (e.g. ``{"spares": {"allowMismatched": True}}``)."""
        self.dir = os.path.abspath(workdir)
        os.makedirs(self.dir, exist_ok=True)
        self.node = node
        self.nodes = [node] + list(extra_nodes)
        self.coord_socket = f"unix:{self.dir}/coord.sock"
        self.daemon_sockets = {n: f"unix:{self.dir}/{n}.sock" for n in self.nodes}
        self.store_sockets = {n: f"unix:{self.dir}/store-{n}.sock" for n in self.nodes}
        self.replica_addrs = {n: f"127.0.0.1:{free_port()}" for n in self.nodes}
        self.cache_dirs = {n: os.path.join(self.dir, f"compile-cache-{n}") for n in self.nodes}
        self.daemon_socket = self.daemon_sockets[node]
        self.store_socket = self.store_sockets[node]
        self.api = f"127.0.0.1:{free_port()}"
        self.policy_path = os.path.join(self.dir, "policy.json")
        with open(self.policy_path, "w") as f:
            json.dump({"outcomesInOrder": list(outcomes), "engines": engines or [], "cover": {"enabled": cover},
                       **(policy_extra or {})}, f)
        self.heartbeat_ms = heartbeat_ms
        self.store_slots = store_slots
        self.store_budget = store_budget
        self.ack_timeout_ms = ack_timeout_ms
        self.standby = standby
        self.node_args = list(node_args or [])
        self.node_extra = dict(node_extra or {})
        self.coord_env = coord_env or {}
        self.procs: dict[str, subprocess.Popen] = {}
        self._logs = []

    def _run(self, name: str, args: list[str], env: dict | None = None) -> None:
        log = open(os.path.join(self.dir, f"{name}.log"), "w")  # noqa: SIM115
        self._logs.append(log)
        e = None
        if env:
            e = dict(os.environ)
            e.update(env)
        self.procs[name] = subprocess.Popen(args, stdout=log, stderr=subprocess.STDOUT, env=e)

    def start(self) -> "ControlPlane":
        for n in self.nodes:
            self._run("store" if n == self.node else f"store-{n}",
                      [binary("everserve-store"), "--socket", self.store_sockets[n], "--data-dir",
                       os.path.join(self.dir, "store" if n == self.node else f"store-{n}"), "--slots",
                       str(self.store_slots), "--budget-bytes", str(self.store_budget), "--replica-listen",
                       self.replica_addrs[n], "--compile-cache-dir", self.cache_dirs[n]])
        coord = [binary("everserve-coord"), "--listen", self.coord_socket, "--policy", self.policy_path,
                 "--spec-store", os.path.join(self.dir, "spec"), "--lease", os.path.join(self.dir, "lease"),
                 "--api-addr", self.api]
        self._run("coord", coord, self.coord_env)
        wait_listening(self.coord_socket)
        if self.standby:
            self._run("coord-standby", coord)  # blocks on the lease until the first one exits
        for n in self.nodes:
            self._run("node" if n == self.node else f"node-{n}",
                      [binary("everserve-node"), "--node", n, "--socket", self.daemon_sockets[n],
                       "--coordinator", self.coord_socket, "--heartbeat-ms", str(self.heartbeat_ms),
                       "--ack-timeout-ms", str(self.ack_timeout_ms), "--mirror-socket", self.store_sockets[n],
                       "--replica-address", self.replica_addrs[n]] + self.node_args + list(self.node_extra.get(n, [])),
                      {"EVERSERVE_COMPILE_CACHE": self.cache_dirs[n]})
        for n in self.nodes:
            wait_listening(self.store_sockets[n])
            wait_listening(self.daemon_sockets[n])
        wait_listening(self.api)
        return self

    def get(self, path: str) -> dict:
        import http.client

        host, _, port = self.api.rpartition(":")
        c = http.client.HTTPConnection(host, int(port), timeout=5)
        c.request("GET", path)
        body = c.getresponse().read()
        c.close()
        return json.loads(body)

    def request(self, method: str, path: str, body: dict | None = None) -> tuple[int, dict]:
        """An operator API call: (status, JSON answer)."""
        import http.client

        host, _, port = self.api.rpartition(":")
        c = http.client.HTTPConnection(host, int(port), timeout=5)
        c.request(method, path, body=json.dumps(body) if body is not None else None,
                  headers={"Content-Type": "application/json"})
        r = c.getresponse()
        data = r.read()
        c.close()
        return r.status, json.loads(data) if data else {}

    def engine_view(self, name: str) -> dict:
        return self.get(f"/v1/engines/{name}")

    def wait_spares(self, engine: str, n: int, timeout_s: float = 600.0) -> None:
        deadline = time.monotonic() + timeout_s
        while time.monotonic() < deadline:
            try:
                if len(self.engine_view(engine)["status"]["spares"]) >= n:
                    return
            except (OSError, KeyError, ValueError):
                pass
            time.sleep(0.1)
        raise TimeoutError(f"{n} spare(s) of {engine} did not register")

    def log(self, name: str) -> str:
        with open(os.path.join(self.dir, f"{name}.log")) as f:
            return f.read()

    def stop(self) -> None:
        for p in reversed(list(self.procs.values())):
            if p.poll() is None:
                p.terminate()
        for p in self.procs.values():
            try:
                p.wait(timeout=5)
            except subprocess.TimeoutExpired:
                p.kill()
                p.wait()
        for f in self._logs:
            f.close()

    def __enter__(self) -> "ControlPlane":
        try:
            return self.start()
        except BaseException:
            self.stop()  # a binary that came up before the failure must not outlive the test
            raise

    def __exit__(self, *exc) -> None:
        self.stop()
