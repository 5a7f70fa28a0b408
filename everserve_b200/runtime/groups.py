"""Process groups per membership epoch, the pipeline transport, and the swap between them.

Every epoch has its own groups. They are built from the engine's rendezvous store under the prefix
``e<epoch>/``, so a spare that takes a lost rank forms the new groups with the survivors without
any process restarting and without the default process group (whose membership cannot change).
Ranks keep their logical positions across epochs: a spare holds the rank it took.

* :class:`EpochGroups` - one epoch's groups for one rank: its column's pipeline group (sends and
  receives between stages) and its stage's tensor-parallel group. gloo on the CPU, NCCL on GPUs.
* :class:`Exchange` - the pipeline transport: a stage's output (hidden state and residual, one
  ``[2, n, hidden]`` tensor) goes to the same column of the next stage.
* :class:`GroupCollective` - the model's tensor-parallel all-reduce / all-gather over an epoch's
  group (the library path; the GPU serving path uses the fused peer-memory kernels instead).
* :class:`SwappableGroups` - holds the live epoch's groups, refuses further use of them when a
  change is staged (a send or receive to a dead peer ends with an error, never a hang: gloo
  reports the closed connection, NCCL groups are aborted), and swaps in the next epoch's groups
  at the step boundary.

Reference parity: the group swap of core/everserve/comm/collective.py and the pipeline transport
of core/everserve/comm/exchange.py (here: c10d groups keyed by epoch instead of swapped pointers).
"""

from __future__ import annotations

import datetime
import threading
import time

import torch
import torch.distributed as dist

from .layout import ParallelLayout


class GroupRefused(RuntimeError):
    """The group belongs to an epoch a membership change has ended."""


def _make_pg(store, prefix: str, rank: int, size: int, device: torch.device, timeout_s: float):
    ps = dist.PrefixStore(prefix, store)
    timeout = datetime.timedelta(seconds=timeout_s)
    if device.type == "cuda":
        opts = dist.ProcessGroupNCCL.Options()
        opts._timeout = timeout
        return dist.ProcessGroupNCCL(ps, rank, size, opts)
    return dist.ProcessGroupGloo(ps, rank, size, timeout)


class EpochGroups:
    """`pipe`: the rank's column across the stages (group rank = stage), for the pipeline's sends
    and receives; `tp`: the rank's stage (group rank = column). A pipe group formed ahead of the
    change (a cover group over the same members) can be handed in as `pipe`."""

    def __init__(self, store, epoch: int, rank: int, layout: ParallelLayout, device: torch.device,
                 timeout_s: float = 30.0, pipe=None):
        self.epoch, self.rank, self.layout, self.device = epoch, rank, layout, device
        self.world_size = layout.world
        pp = layout.pipeline_parallel
        self.adopted = pipe is not None
        self.pipe = pipe
        if self.pipe is None and pp > 1:
            col = layout.column(rank) + layout.replica(rank) * layout.tensor_parallel
            self.pipe = _make_pg(store, f"e{epoch}/pipe{col}/", layout.stage(rank), pp, device, timeout_s)
        tp = layout.tensor_parallel
        self.tp = None
        if tp > 1:
            stage = layout.stage(rank) + layout.replica(rank) * layout.pipeline_parallel
            self.tp = _make_pg(store, f"e{epoch}/tp{stage}/", layout.column(rank), tp, device, timeout_s)

    def abort(self) -> None:
        for pg in (self.pipe, self.tp):
            if pg is None:
                continue
            try:
                if hasattr(pg, "abort"):
                    pg.abort()
                elif hasattr(pg, "shutdown"):
                    pg.shutdown()
            except Exception:  # noqa: BLE001 - best effort on a dead group
                pass


class SwappableGroups:
    """The live epoch's groups; refused while a change is staged, replaced at the boundary.

    A refused epoch's groups are released beside the change, on a thread, within
    `release_bound_s`: an abort that does not return by then (a communicator stuck on a dead peer)
    is a leak, reported through `on_leak(release, seconds, leaked_total)`; the process keeps
    serving, and the control plane retires it by notice at a later boundary."""

    def __init__(self, store, rank: int, layout: ParallelLayout, device: torch.device, timeout_s: float = 30.0,
                 release_bound_s: float = 10.0, on_leak=None):
        self.store, self.rank, self.layout, self.device, self.timeout_s = store, rank, layout, device, timeout_s
        self.current: EpochGroups | None = None
        self.refused = threading.Event()
        self._lock = threading.Lock()
        self.release_bound_s = release_bound_s
        self.on_leak = on_leak
        self.leaked = 0

    def _release(self, g: "EpochGroups", what: str) -> None:
        """Abort `g` beside the caller, bounded; a release past the bound is reported as a leak."""
        done = threading.Event()

        def run():
            g.abort()
            done.set()

        def watch():
            t0 = time.monotonic()
            if not done.wait(self.release_bound_s):
                self.leaked += 1
                if self.on_leak is not None:
                    self.on_leak(what, time.monotonic() - t0, self.leaked)

        threading.Thread(target=run, name=f"release-e{g.epoch}", daemon=True).start()
        threading.Thread(target=watch, name=f"release-watch-e{g.epoch}", daemon=True).start()

    def form(self, epoch: int, rank: int | None = None, pipe=None) -> EpochGroups:
        """Build the epoch's groups (a rendezvous with every member of the epoch), adopting `pipe`
        when a pre-formed pipeline group over the epoch's members is at hand."""
        if rank is not None:
            self.rank = rank
        g = EpochGroups(self.store, epoch, self.rank, self.layout, self.device, self.timeout_s, pipe=pipe)
        with self._lock:
            old, self.current = self.current, g
            self.refused.clear()
        if old is not None:
            self._release(old, f"epoch {old.epoch} groups")
        return g

    def refuse(self) -> None:
        """A change is staged: no further use of the live groups (NCCL groups are aborted)."""
        self.refused.set()
        with self._lock:
            g = self.current
        if g is not None and self.device.type == "cuda":
            self._release(g, f"epoch {g.epoch} groups (refused)")

    def live(self) -> EpochGroups:
        if self.refused.is_set() or self.current is None:
            raise GroupRefused("the groups of this epoch were refused by a membership change")
        return self.current


def _wait(groups: "SwappableGroups", work) -> None:
    """Wait for a c10d operation. One with a dead peer ends with an error: on gloo when the kernel
    closes the peer's sockets, on NCCL when a change refuses the groups (they are aborted). gloo's
    point-to-point work only completes inside wait(), so it cannot be polled instead."""
    work.wait()


class Exchange:
    """Pipeline transport between the same column of adjacent stages."""

    def __init__(self, groups: SwappableGroups, hidden: int, dtype: torch.dtype):
        self.groups, self.hidden, self.dtype = groups, hidden, dtype

    def send_hidden(self, hidden: torch.Tensor, residual: torch.Tensor) -> None:
        g = self.groups.live()
        buf = torch.stack([hidden.to(self.dtype), residual.to(self.dtype)]).contiguous()
        _wait(self.groups, g.pipe.send([buf], g.layout.stage(g.rank) + 1, 0))

    def recv_hidden(self, n: int) -> tuple[torch.Tensor, torch.Tensor]:
        g = self.groups.live()
        buf = torch.empty(2, n, self.hidden, dtype=self.dtype, device=g.device)
        _wait(self.groups, g.pipe.recv([buf], g.layout.stage(g.rank) - 1, 0))
        return buf[0], buf[1]


class GroupCollective:
    """Tensor-parallel all-reduce / all-gather over the live epoch's stage group."""

    def __init__(self, groups: SwappableGroups):
        self.groups = groups

    def all_reduce(self, t: torch.Tensor) -> torch.Tensor:
        g = self.groups.live()
        if g.tp is not None:
            _wait(self.groups, g.tp.allreduce([t]))
        return t

    def all_gather(self, t: torch.Tensor) -> torch.Tensor:
        g = self.groups.live()
        if g.tp is None:
            return t
        t = t.contiguous()
        parts = [torch.empty_like(t) for _ in range(g.layout.tensor_parallel)]
        _wait(self.groups, g.tp.allgather([parts], [t]))
        return torch.cat(parts, dim=-1)
