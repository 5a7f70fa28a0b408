"""A spare its node's daemon launched: fetch the engine's start-up record, then stand for a rank.

    (launched by everserve-node for a LaunchSpare; the environment names the engine, the rank it
     stands for, the device, the daemon's socket, the node and the store's socket)
    python -m everserve_b200.serving.spare

The spare does not know how the engine was started. It asks its daemon for the start-up record
(``ReplayAsk``; the daemon stamps where the answer must come back to and the coordinator relays
the ask to the engine's head), and the head answers with a ``ReplayOffer`` carrying the record as
JSON: the model and engine configuration, the rendezvous address, the slot region and a row of
it for this spare. With that the process builds the rank's shard, restores nothing yet, and
registers as ``ROLE_SPARE`` (``everserve_b200.serving.rank``); the daemon restarts it with a
backoff if it exits before it takes a rank.

Reference parity: spare_main of adapters/vllm/everserve_vllm/spare_main.py:43-984 (policy and
discovery, replay fetch, stand, register, wait for the join) and the start-up record of
replay.py:65-462 (here one JSON record instead of the engine core's recorded broadcasts).
"""

from __future__ import annotations

import json
import os
import sys
import time

from ..contract.daemon import _Link
from ..proto import signals as sp


def fetch_startup(daemon: str, engine: str, rank: int, timeout_s: float = 120.0) -> dict:
    """Ask the engine's head for its start-up record; retries until the head answers."""
    deadline = time.monotonic() + timeout_s
    while True:
        link = _Link(daemon, timeout_s=min(10.0, timeout_s))
        try:
            link.send(sp.Signal(replay_ask=sp.ReplayAsk(engine=engine, rank=rank)))
            link.sock.settimeout(5.0)
            while True:
                sig = link.recv()
                if sig.WhichOneof("kind") == "replay_offer" and sig.replay_offer.engine == engine:
                    return json.loads(sig.replay_offer.handle)
        except (TimeoutError, OSError, ConnectionError):
            if time.monotonic() > deadline:
                raise TimeoutError(f"no start-up record from {engine}'s head within {timeout_s} s") from None
        finally:
            link.close()
        time.sleep(0.5)


def main() -> int:
    engine = os.environ["EVERSERVE_ENGINE"]
    rank_s = os.environ.get("EVERSERVE_SPARE_RANK", "any")
    if not rank_s.isdigit():
        print("a spare launched by a daemon stands for one rank (EVERSERVE_SPARE_RANK)", file=sys.stderr)
        return 2
    rank = int(rank_s)
    daemon = os.environ["EVERSERVE_SOCKET"]
    rec = fetch_startup(daemon, engine, rank)
    from .rank import main as rank_main

    argv = list(rec["args"]) + ["--role", "spare", "--rank", str(rank), "--daemon", daemon,
                                "--node", os.environ.get("EVERSERVE_NODE", "")]
    store = os.environ.get("EVERSERVE_MIRROR_SOCKET", "")
    if store:
        argv += ["--store", store]
    if rec.get("row") is not None:
        argv += ["--row", str(rec["row"])]
    if rec.get("gpu"):
        argv += ["--device", f"cuda:{os.environ.get('EVERSERVE_DEVICE', '0')}"]
    return rank_main(argv)


if __name__ == "__main__":
    sys.exit(main())
