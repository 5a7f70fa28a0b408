"""The paths, group and environment a node's daemon, store and engine processes share.

The daemon's socket directory, the shared-memory directory of the store's tables and the slot
region, the compile-cache directory, the node group that owns them (files are group-read/write so
every engine process on the node can map them), and the pod fragments (security context, env,
volumes, mounts) a Kubernetes renderer puts on engine pods.

Reference parity: core/everserve/podcontract.py:21-98 (same paths, group id and modes, so pods built
for either side share a node).
"""

from __future__ import annotations

import os

DAEMON_DIR = "/run/everserve"
DAEMON_SOCKET = f"{DAEMON_DIR}/node.sock"
SHM_DIR = "/dev/shm/everserve"
SHM_DIR_ENV = "EVERSERVE_SHM_DIR"
COMPILE_CACHE_DIR = "/var/lib/everserve/compile-cache"
COMPILE_CACHE_ENV = "EVERSERVE_COMPILE_CACHE"
NODE_GID = 64000
SHARED_MODE = 0o660
NODE_ENV = "EVERSERVE_NODE"


def shm_dir() -> str:
    return os.environ.get(SHM_DIR_ENV, SHM_DIR)


def make_shared(path: str, size: int) -> None:
    """Create (or grow) a file of `size` bytes that every process of the node group may map."""
    fd = os.open(path, os.O_RDWR | os.O_CREAT, SHARED_MODE)
    try:
        if os.fstat(fd).st_size < size:
            os.ftruncate(fd, size)
        try:
            os.fchmod(fd, SHARED_MODE)
            if os.getuid() == 0:
                os.fchown(fd, -1, NODE_GID)
        except OSError:
            pass
    finally:
        os.close(fd)


def security_context() -> dict:
    return {"runAsGroup": NODE_GID, "fsGroup": NODE_GID, "supplementalGroups": [NODE_GID]}


def env() -> list[dict]:
    return [{"name": NODE_ENV, "valueFrom": {"fieldRef": {"fieldPath": "spec.nodeName"}}},
            {"name": "EVERSERVE_DAEMON_SOCKET", "value": DAEMON_SOCKET},
            {"name": SHM_DIR_ENV, "value": SHM_DIR},
            {"name": COMPILE_CACHE_ENV, "value": COMPILE_CACHE_DIR}]


def volumes() -> list[dict]:
    return [{"name": "everserve-run", "hostPath": {"path": DAEMON_DIR, "type": "Directory"}},
            {"name": "everserve-shm", "hostPath": {"path": SHM_DIR, "type": "DirectoryOrCreate"}},
            {"name": "everserve-cache", "hostPath": {"path": COMPILE_CACHE_DIR, "type": "DirectoryOrCreate"}}]


def mounts() -> list[dict]:
    return [{"name": "everserve-run", "mountPath": DAEMON_DIR},
            {"name": "everserve-shm", "mountPath": SHM_DIR},
            {"name": "everserve-cache", "mountPath": COMPILE_CACHE_DIR}]
