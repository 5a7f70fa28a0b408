"""The indirection captured code reads, and the stand-in a spare captures against.

A CUDA graph captures the kernels of a step, including its collectives, with their arguments.
The collectives here take their members, order and peer tables from device memory that the
collective object owns, so a membership change rewrites those tables and the same graph keeps
working: :class:`GroupHandle` is the host-side object code asks for "the current group", and the
swap happens under it. A spare has no peers while it stands; it captures its graphs against
:class:`LocalStandIn`, which has the collective's interface and computes as a group of one, and
the real collective replaces it when the spare takes a rank (the graphs are captured again at the
take only if the kernel arguments differ).

Reference parity: GroupHandle / LocalStandIn of core/everserve/comm/handle.py:23-63.
"""

from __future__ import annotations

import threading

import torch


class LocalStandIn:
    """A group of one with the collective's interface."""

    size = 1
    rank = 0

    def all_reduce(self, t: torch.Tensor) -> torch.Tensor:
        return t

    def all_gather(self, t: torch.Tensor) -> torch.Tensor:
        return t

    def linear_allreduce(self, ops, x, w, residual=None):
        return ops.linear(x, w, residual=residual)


class GroupHandle:
    def __init__(self, initial=None):
        self._lock = threading.Lock()
        self._current = initial if initial is not None else LocalStandIn()
        self.generation = 0

    @property
    def current(self):
        return self._current

    def swap(self, new) -> object:
        with self._lock:
            old, self._current = self._current, new
            self.generation += 1
        return old

    # the collective interface, forwarded (what the model's TPGroup calls)
    def all_reduce(self, t):
        return self._current.all_reduce(t)

    def all_gather(self, t):
        return self._current.all_gather(t)

    def __getattr__(self, name):
        return getattr(self._current, name)
