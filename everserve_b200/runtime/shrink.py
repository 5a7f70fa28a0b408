"""A process group that can shrink to its survivors.

``shrink(lost, epoch)`` replaces the group by its survivors' group; every survivor calls it with the
same arguments, and ranks are renumbered densely in the old order. Two ways:

* NCCL shrink: for an NCCL group that was not formed over a store (``from_group``), the survivors
  split the communicator with the lost ranks excluded and the old one aborted
  (``ncclCommShrink`` through ``torch.distributed.shrink_group`` with ``SHRINK_ABORT``), which
  needs no rendezvous at all;
* recreate: otherwise, or when the NCCL shrink fails (the failure is kept in ``shrink_failure``),
  the old group is aborted (NCCL) so nothing waits on the dead member, and the survivors form a new
  group over the rendezvous store under an epoch-keyed prefix.

``method`` records which one formed the current group. This is the SHRINK outcome's group operation
(the CPU reference tier uses it; the GPU product path is REPLACE).

Reference parity: ShrinkableGroup of core/everserve/comm/group.py:29-155 (both methods, the same
fallback order).
"""

from __future__ import annotations

import datetime

import torch.distributed as dist

RECREATE = "recreate"
NCCL_SHRINK = "nccl_shrink"


class ShrinkableGroup:
    def __init__(self, store, members: list[int], me: int, backend: str = "gloo", timeout_s: float = 30.0,
                 epoch: int = 0):
        self.store, self.backend, self.timeout_s = store, backend, timeout_s
        self.me = me
        self.members = list(members)
        self.epoch = epoch
        self.method = RECREATE
        self.shrink_failure: str | None = None
        self.pg = self._form() if store is not None else None

    @classmethod
    def from_group(cls, pg, members: list[int], me: int, backend: str = "nccl", timeout_s: float = 30.0,
                   store=None) -> "ShrinkableGroup":
        """Wrap a group made elsewhere (no store of its own: an NCCL group shrinks in place; `store`
        is kept for the recreate fallback)."""
        self = cls(None, members, me, backend, timeout_s)
        self.pg = pg
        self.store = store
        self.method = "given"
        return self

    def _form(self):
        prefix = f"shrink/e{self.epoch}/" + ",".join(map(str, self.members)) + "/"
        ps = dist.PrefixStore(prefix, self.store)
        rank, size = self.members.index(self.me), len(self.members)
        t = datetime.timedelta(seconds=self.timeout_s)
        if self.backend == "nccl":
            opts = dist.ProcessGroupNCCL.Options()
            opts._timeout = t
            return dist.ProcessGroupNCCL(ps, rank, size, opts)
        return dist.ProcessGroupGloo(ps, rank, size, t)

    @property
    def rank(self) -> int:
        return self.members.index(self.me)

    @property
    def size(self) -> int:
        return len(self.members)

    def all_reduce(self, t):
        self.pg.allreduce([t]).wait()
        return t

    def all_reduce_async(self, t):
        """The collective's work handle (``is_completed`` / ``wait``)."""
        return self.pg.allreduce([t])

    def _abort(self) -> None:
        if self.pg is not None and hasattr(self.pg, "abort"):
            try:
                self.pg.abort()
            except Exception:  # noqa: BLE001 - an abort that fails must not stop recovery
                pass

    def shrink(self, lost, epoch: int) -> None:
        lost = set(lost)
        stray = lost - set(self.members)
        if stray:
            raise ValueError(f"ranks {sorted(stray)} are not members of {self.members}")
        if self.me in lost:
            raise ValueError(f"member {self.me} is among the lost")
        excluded = [self.members.index(m) for m in self.members if m in lost]
        survivors = [m for m in self.members if m not in lost]
        self.shrink_failure = None
        if self.backend == "nccl" and hasattr(dist, "shrink_group") and self.method != RECREATE:
            try:
                from torch.distributed import distributed_c10d as c10d

                pg = dist.shrink_group(excluded, group=self.pg, shrink_flags=c10d.SHRINK_ABORT)
                self.pg, self.members, self.epoch, self.method = pg, survivors, epoch, NCCL_SHRINK
                return
            except Exception as e:  # noqa: BLE001 - fall back to recreate, and say why
                self.shrink_failure = f"{type(e).__name__}: {e}"
        if self.store is None:
            raise RuntimeError(f"no store to re-form the group over ({self.shrink_failure or 'not an NCCL group'})")
        self._abort()
        self.members = survivors
        self.epoch = epoch
        self.pg = self._form()
        self.method = RECREATE
