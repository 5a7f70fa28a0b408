"""The engine's plugin surface: what a fault-tolerant deployment hooks into a serving engine.

The reference is a vLLM plugin whose single entry point, called in every engine process, installs
a listed set of patches on vLLM (adapters/vllm/everserve_vllm/__init__.py:86-140,
adapters/vllm/everserve_vllm/patches.py). This framework owns its engine, so the hook points are
attributes of :class:`everserve_b200.engine.Engine` rather than patched internals, and
:func:`register` installs them through the same kind of ledger:

  * ``executor``   the executor that runs step plans (a multi-process executor with spares);
  * ``connector``  the KV connector called around each step (begin / end / finished / commit);
  * ``step-hook``  a wrapper around the step function that completes membership changes at the
                   step boundary (``serving.executor.failover``);
  * ``collective`` the tensor-parallel collective the row-parallel linears go through (set on the
                   engine's ranks, not the head: see ``serving.rank``).

Every patch is named, applied at most once per engine and listed on the engine afterwards
(``engine.plugin_patches``), so a process can report exactly what it runs.
"""

from __future__ import annotations

import faulthandler
import os
import signal
from dataclasses import dataclass
from typing import Callable

STACKS_SIGNAL = signal.SIGUSR1
"""Dumps every thread's stack in an engine process (the daemon's stack request, ``kill -USR1``)."""


def prepare_engine_process() -> None:
    """Settings every process of a fault-tolerant engine needs before its ranks start: the stacks
    signal, and NCCL's own error handling off (a survivor must not tear itself down when a peer
    dies; the runtime swaps its groups instead). Ranks inherit the environment from the head."""
    try:
        faulthandler.register(STACKS_SIGNAL, all_threads=True)
    except (AttributeError, ValueError, RuntimeError):
        pass
    os.environ.setdefault("TORCH_NCCL_ASYNC_ERROR_HANDLING", "0")
    os.environ.setdefault("TORCH_NCCL_ENABLE_MONITORING", "0")


@dataclass(frozen=True)
class Patch:
    """One hook point: the engine attribute it sets and what it does there."""

    name: str
    attribute: str
    what: str


PATCHES = (
    Patch("executor", "executor", "runs plans on rank processes that a spare can replace"),
    Patch("connector", "connector", "commits each step's KV rows to the node's store"),
    Patch("step-hook", "step_fn", "completes a membership change at the step boundary"),
)


def register(engine, *, executor=None, connector=None, step_hook: Callable | None = None,
             prepare: bool = True) -> list[str]:
    """Install the given hooks on `engine`; returns the names of the patches now applied.

    ``step_hook`` defaults to the failover hook when the executor (given, or the engine's) is the
    multi-process executor. Installing a patch twice is refused: a second step hook around the
    first would complete a change twice."""
    if prepare:
        prepare_engine_process()
    applied: list[str] = list(getattr(engine, "plugin_patches", []))

    def mark(name: str) -> None:
        if name in applied:
            raise RuntimeError(f"plugin patch {name!r} is already installed on this engine")
        applied.append(name)

    if executor is not None:
        mark("executor")
        engine.executor = executor
    if connector is not None:
        mark("connector")
        engine.connector = connector
    ex = engine.executor
    if step_hook is None:
        from ..serving.executor import MultiprocExecutor, failover

        if isinstance(ex, MultiprocExecutor) and "step-hook" not in applied:
            step_hook = failover(ex, engine)
    if step_hook is not None:
        mark("step-hook")
        engine.wrap_step(step_hook)
    engine.plugin_patches = applied
    return list(applied)


__all__ = ["PATCHES", "Patch", "STACKS_SIGNAL", "prepare_engine_process", "register"]
