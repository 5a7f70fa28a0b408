"""An exact committed-KV store for the reference tier, over multiprocessing connections.

``ExactStore`` serves, in a thread, what ranks commit: KV rows keyed by (layer, KV head, sequence)
and by the step that wrote them. Rows are kept as the exact tensors sent (no conversion). A
commit of a step the store holds replaces it (a re-run step writes the same rows again, never
twice); a commit from an epoch older than the store has seen for a rank is refused. ``restore``
returns a lost rank's rows for the heads a survivor absorbs, up to a step when one is given (a
step the survivors did not accept is left out). ``LoopbackCommittedKV`` is a rank's client.

Reference parity: core/everserve/reference/store.py:40-246 and committed.py:22-79 (a synchronous
exact store for the CPU tier; the product path uses the C++ store).
"""

from __future__ import annotations

import threading
from multiprocessing.connection import Client, Listener

import torch


class ExactStore:
    def __init__(self, address=("127.0.0.1", 0), authkey: bytes = b"everserve-reference"):
        self._listener = Listener(address, authkey=authkey)
        self.address = self._listener.address
        self.authkey = authkey
        # (layer, head, seq) -> {step: [n, 2, d]}
        self.rows: dict[tuple[int, int, int], dict[int, torch.Tensor]] = {}
        self.owner: dict[tuple[int, int, int], int] = {}
        self.epochs: dict[int, int] = {}
        self.steps: dict[int, int] = {}
        self._lock = threading.Lock()
        self._stop = False
        threading.Thread(target=self._accept, daemon=True).start()

    def _accept(self) -> None:
        while not self._stop:
            try:
                conn = self._listener.accept()
            except OSError:
                return
            threading.Thread(target=self._serve, args=(conn,), daemon=True).start()

    def _serve(self, conn) -> None:
        while True:
            try:
                op, args = conn.recv()
            except (EOFError, OSError):
                return
            try:
                conn.send(("ok", getattr(self, "_" + op)(*args)))
            except Exception as e:  # noqa: BLE001 - the client raises it
                conn.send(("error", str(e)))

    def _commit(self, rank: int, epoch: int, step: int, rows: dict) -> int:
        with self._lock:
            if epoch < self.epochs.get(rank, 0):
                raise ValueError(f"stale epoch {epoch} for rank {rank}")
            self.epochs[rank] = epoch
            for key, new in rows.items():
                self.rows.setdefault(key, {})[step] = new.clone()
                self.owner[key] = rank
            self.steps[rank] = step
        return step

    def _restore(self, heads: list, upto_step: int | None = None) -> dict:
        want = set(heads)
        out = {}
        with self._lock:
            for k, by_step in self.rows.items():
                if k[1] not in want:
                    continue
                parts = [by_step[s] for s in sorted(by_step) if upto_step is None or s <= upto_step]
                if parts:
                    out[k] = torch.cat(parts)
        return out

    def _moved(self, heads: list, rank: int) -> int:
        """The heads now belong to `rank` (its later commits extend their rows)."""
        with self._lock:
            for k in self.rows:
                if k[1] in set(heads):
                    self.owner[k] = rank
        return 0

    def close(self) -> None:
        self._stop = True
        self._listener.close()


class LoopbackCommittedKV:
    """A rank's client of the ExactStore (commit per step; restore of absorbed heads)."""

    def __init__(self, address, authkey: bytes = b"everserve-reference"):
        self._conn = Client(address, authkey=authkey)
        self._lock = threading.Lock()

    def _call(self, op: str, *args):
        with self._lock:
            self._conn.send((op, args))
            status, value = self._conn.recv()
        if status != "ok":
            raise RuntimeError(value)
        return value

    def commit(self, rank: int, epoch: int, step: int, rows: dict) -> int:
        return self._call("commit", rank, epoch, step, rows)

    def restore(self, heads, upto_step: int | None = None) -> dict:
        return self._call("restore", list(heads), upto_step)

    def close(self) -> None:
        self._conn.close()
