"""The engine's KV connector over a committed-KV store: every step's rows and counts committed.

``Engine`` calls ``begin_step`` / ``end_step`` / ``finished`` around each step (its plugin surface);
multi-step decoding calls ``commit_rows`` once per decode step it runs on the device. A commit
launches the gather of the step's rows on the committed-KV object's side stream behind the step's
kernels and hands the store request to its sender thread; the connector then fences the commit
``depth`` steps back, so the step loop never waits for the store unless it runs more than
``depth`` steps ahead of its acknowledgements. This is the per-rank commit path of the serving
ranks (``serving.rank``) in a form a single-process engine can use.

Reference parity: the KV connector's per-step save/commit of
adapters/vllm/everserve_vllm/connector.py over core/everserve/state/mirror.py:645-706.
"""

from __future__ import annotations

from typing import Mapping

from .mirror import DEPTH


class StoreConnector:
    def __init__(self, ckv, block_size: int, epoch: int = 0, depth: int = DEPTH):
        self.ckv = ckv
        self.block_size = block_size
        self.epoch = epoch
        self.depth = depth
        self._issued: list[int] = []
        self.commits = 0

    # ---- the engine's hooks ----------------------------------------------------------------------
    def begin_step(self, plan, scheduler) -> None:
        """Nothing to do before a step: rows are gathered after the step's kernels."""

    def end_step(self, plan, scheduler) -> None:
        counts = {r.req_id: r.start_pos + len(r.token_ids) for r in plan.reqs}
        slots = [s for row in plan.slots(self.block_size) for s in row]
        self.commit_rows(plan.step, counts, slots)

    def finished(self, req_id: str) -> None:
        self.ckv.finished(req_id)

    # ---- commits -----------------------------------------------------------------------------
    def commit_rows(self, step: int, counts: Mapping[str, int], slots: list[int]) -> None:
        """Commit one step (its rows at `slots`, the requests' computed counts), then fence the
        commit `depth` steps back."""
        self.ckv.commit(self.epoch, step, counts, slots)
        self.commits += 1
        self._issued.append(step)
        if len(self._issued) > self.depth:
            self.ckv.fence(self._issued[-1 - self.depth])
        del self._issued[: -(self.depth + 1)]

    def drain(self, timeout_s: float = 30.0) -> None:
        """Wait until every commit issued so far is acknowledged."""
        if self._issued:
            self.ckv.fence(self._issued[-1], timeout_s=timeout_s)

    def decode_hook(self, plan, k: int):
        """The per-step commit callback of a k-step device decode from `plan` (step i's rows are
        the position start_pos + i of every request; the tables already cover them)."""
        bs = self.block_size
        starts = [(r.req_id, r.start_pos, list(r.block_table)) for r in plan.reqs]
        base = plan.step

        def after_step(i: int) -> None:
            counts = {rid: p + 1 + i for rid, p, _ in starts}
            slots = [bt[(p + i) // bs] * bs + (p + i) % bs for _, p, bt in starts]
            self.commit_rows(base + i, counts, slots)

        return after_step

    def close(self) -> None:
        self.drain()
        self.ckv.close()
