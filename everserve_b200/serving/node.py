"""The node role: starts and supervises an engine's ranks on a node other than the head's.

    EVERSERVE_SOCKET=unix:/run/everserve/node.sock EVERSERVE_NODE=n1 \
    EVERSERVE_MIRROR_SOCKET=unix:/run/everserve/store.sock \
    python -m everserve_b200.serving.node --engine e0 --ranks 4,5,6,7 [--devices 0,1,2,3]

The agent asks the engine's head for its start-up record through the control plane (the same
ReplayAsk / ReplayOffer a daemon-launched spare uses), then starts one rank process per position
on this node, linked to its node's daemon and store, and waits on them. It forwards SIGTERM and
exits once they all have. A rank that dies is reported by its daemon (its connection ends) and
the engine's failover takes it from there; the agent does not restart workers.

Reference parity: the node role of adapters/vllm/everserve_vllm/node.py and node_main.py (an
executor on each non-head node that starts its ranks and releases them); this agent is a launcher
around this framework's rank processes.
"""

from __future__ import annotations

import argparse
import os
import signal
import subprocess
import sys

from .spare import fetch_startup


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--engine", required=True)
    p.add_argument("--ranks", required=True, help="comma-separated rank positions on this node")
    p.add_argument("--devices", default="", help="comma-separated GPU indices, one per rank")
    p.add_argument("--daemon", default=os.environ.get("EVERSERVE_SOCKET", ""))
    p.add_argument("--store", default=os.environ.get("EVERSERVE_MIRROR_SOCKET", ""))
    p.add_argument("--node", default=os.environ.get("EVERSERVE_NODE", ""))
    p.add_argument("--threads", type=int, default=0)
    a = p.parse_args(argv)
    ranks = [int(r) for r in a.ranks.split(",") if r]
    devices = [int(d) for d in a.devices.split(",") if d] or list(range(len(ranks)))
    rec = fetch_startup(a.daemon, a.engine, ranks[0])
    env = dict(os.environ)
    env["EVERSERVE_CARRIER_TOKEN"] = rec["token"]
    procs = []
    for r, dev in zip(ranks, devices):
        cmd = [sys.executable, "-m", "everserve_b200.serving.rank"] + list(rec["args"]) + [
            "--role", "worker", "--rank", str(r), "--row", str(r), "--daemon", a.daemon, "--node", a.node]
        if a.store:
            cmd += ["--store", a.store]
        if rec.get("gpu"):
            cmd += ["--device", f"cuda:{dev}"]
        if a.threads:
            cmd += ["--threads", str(a.threads)]
        procs.append(subprocess.Popen(cmd, env=env))

    def stop(*_):
        for pr in procs:
            if pr.poll() is None:
                pr.terminate()

    signal.signal(signal.SIGTERM, stop)
    codes = [pr.wait() for pr in procs]
    return 0 if all(c == 0 for c in codes) else 1


if __name__ == "__main__":
    sys.exit(main())
