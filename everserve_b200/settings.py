"""Settings read from the environment, with the defaults the runtime uses.

| variable | default | meaning |
|---|---|---|
| ``EVERSERVE_DETECT_STEPS`` | 3 | a collective waits this many measured step periods before it names late members |
| ``EVERSERVE_DETECT_FLOOR_MS`` | 30 | ... but never less than this |
| ``EVERSERVE_HANG_S`` | 10 | a late member that is alive is hung after this long |
| ``EVERSERVE_BEAT_LIMIT_MS`` | 20 | a member whose heartbeat stands still this long is dead (kernels and detector; 0 off) |
| ``EVERSERVE_POLL_MS`` | 2 | the failure detector's poll period |
| ``EVERSERVE_RELEASE_BOUND_MS`` | 10000 | how long a boundary waits for a refused group's release |
| ``EVERSERVE_STEP_SAMPLE`` | 16 | steps measured before the bound is set from the step period |
| ``EVERSERVE_NODE`` | host name | this node's name in the control plane |

Read where they are used (set by the node daemon for the processes it starts, or by the pod):

| variable | meaning |
|---|---|
| ``EVERSERVE_SOCKET`` | the node daemon's process socket |
| ``EVERSERVE_MIRROR_SOCKET`` | the node's KV store socket |
| ``EVERSERVE_ENGINE`` / ``EVERSERVE_ENGINES`` | the engine (or a pool's engines, comma-separated) a launched spare stands for |
| ``EVERSERVE_SPARE_RANK`` | the rank a launched spare stands for, or ``any`` |
| ``EVERSERVE_POOL`` | the pool a launched spare belongs to |
| ``EVERSERVE_DEVICE`` | the GPU a launched spare runs on |
| ``EVERSERVE_COMPILE_CACHE`` | the node's compile-cache directory (workers publish their build there) |
| ``EVERSERVE_FETCH_COMPILE_CACHE`` | ``1``: a spare takes its build from the compile cache even when one is installed |
| ``EVERSERVE_EVENT_DIR`` | where rank processes write their event logs |
| ``EVERSERVE_DISCOVERY_DIR`` | where daemons write their discovery records |
| ``ES_EXTENSION_PATH`` | a kernel extension to load instead of the in-tree build |
| ``ES_PDL`` | ``0``: launch the decode kernels without programmatic dependent launch |
| ``ES_AR_TWO_SHOT`` / ``ES_NVLS`` | the fused all-reduce's variant: two-shot, or NVLS multicast (``0`` off) |
| ``ES_MOE_ROUTED`` | ``1``: mixture layers route tokens to their experts' owners (the peer-memory all-to-all) |

Reference parity: adapters/vllm/everserve_vllm/settings.py:54-99 (same defaults: 3 steps, a 30 ms
floor, 10 s to hung, a 2 ms poll).
"""

from __future__ import annotations

import os
import socket
from dataclasses import dataclass


def _f(name: str, default: float) -> float:
    v = os.environ.get(name, "")
    try:
        return float(v) if v else default
    except ValueError:
        raise ValueError(f"{name}={v!r} is not a number") from None


@dataclass(frozen=True)
class Settings:
    detect_steps: float = 3.0
    detect_floor_ms: float = 30.0
    hang_s: float = 10.0
    beat_limit_ms: float = 20.0
    poll_ms: float = 2.0
    release_bound_ms: float = 10000.0
    step_sample: int = 16
    node: str = ""

    def bound_ns(self, step_period_s: float) -> int:
        """The collective's wait bound for a measured step period."""
        return int(max(self.detect_steps * step_period_s * 1e3, self.detect_floor_ms) * 1e6)

    def warmup_bound_ns(self) -> int:
        """The bound for naming a late member before the step period is measured (the first
        `step_sample` steps): the hung-member limit, so the one-off costs of first steps (first
        launches, allocator growth, graph captures) do not name a member late. The bound only
        names; a member that dies is named by its heartbeat (`beat_limit_ms`) whatever it is."""
        return int(max(self.hang_s * 1e3, self.detect_floor_ms) * 1e6)


def load() -> Settings:
    return Settings(
        detect_steps=_f("EVERSERVE_DETECT_STEPS", 3.0), detect_floor_ms=_f("EVERSERVE_DETECT_FLOOR_MS", 30.0),
        hang_s=_f("EVERSERVE_HANG_S", 10.0), poll_ms=_f("EVERSERVE_POLL_MS", 2.0),
        beat_limit_ms=_f("EVERSERVE_BEAT_LIMIT_MS", 20.0),
        release_bound_ms=_f("EVERSERVE_RELEASE_BOUND_MS", 10000.0), step_sample=int(_f("EVERSERVE_STEP_SAMPLE", 16)),
        node=os.environ.get("EVERSERVE_NODE", socket.gethostname()))
