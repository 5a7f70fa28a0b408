"""A process group that can shrink to its survivors.

``shrink(lost, epoch)`` ends the old group and forms the survivors' group over the rendezvous store
under an epoch-keyed prefix (every survivor calls it with the same arguments); ranks are renumbered
densely in the old order. On NCCL the old communicator is aborted first so nothing waits on the
dead member. This is the SHRINK outcome's group operation (the CPU reference tier uses it; the GPU
product path is REPLACE).

Reference parity: ShrinkableGroup of core/everserve/comm/group.py:29-155 (recreate-over-a-prefixed-
store variant).
"""

from __future__ import annotations

import datetime

import torch.distributed as dist


class ShrinkableGroup:
    def __init__(self, store, members: list[int], me: int, backend: str = "gloo", timeout_s: float = 30.0,
                 epoch: int = 0):
        self.store, self.backend, self.timeout_s = store, backend, timeout_s
        self.me = me
        self.members = list(members)
        self.epoch = epoch
        self.pg = self._form()

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

    def shrink(self, lost, epoch: int) -> None:
        if hasattr(self.pg, "abort"):
            try:
                self.pg.abort()
            except Exception:  # noqa: BLE001
                pass
        self.members = [m for m in self.members if m not in set(lost)]
        if self.me not in self.members:
            raise ValueError(f"member {self.me} is among the lost")
        self.epoch = epoch
        self.pg = self._form()
