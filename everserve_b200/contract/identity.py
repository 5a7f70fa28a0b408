"""A process's software identity: what a spare must share with the ranks it may replace.

``SoftwareIdentity`` (signals.proto) names the engine build, the kernel extension, torch / CUDA /
driver / NCCL versions, the model and its weights' digest, the KV format, the parallel layout, and a
digest of every setting that changes a step's arithmetic. ``mismatch(a, b)`` lists the fields that
must agree for a spare to take a rank with the exact-replay guarantee (a spare on another build
would produce other tokens); the daemon and the coordinator carry the identity with each
registration so a mismatched spare can be refused before it takes anything.

Reference parity: adapters/vllm/everserve_vllm/identity.py:46-503 (the same message; this
framework fills it from its own engine configuration and kernel extension).
"""

from __future__ import annotations

import hashlib
import json
import os
import subprocess

import torch

from ..proto import signals as sp

_EXACT_FIELDS = ("engine_commit", "torch_version", "cuda_version", "nccl_version", "model", "checkpoint_digest",
                 "quantization", "model_dtype", "kv_format", "layout", "step")


def _repo_commit() -> tuple[str, bool]:
    root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    try:
        head = subprocess.run(["git", "-C", root, "rev-parse", "HEAD"], capture_output=True, text=True, timeout=5)
        dirty = subprocess.run(["git", "-C", root, "status", "--porcelain", "--untracked-files=no"],
                               capture_output=True, text=True, timeout=5)
        return head.stdout.strip(), bool(dirty.stdout.strip())
    except (OSError, subprocess.SubprocessError):
        return "", False


def extension_digest() -> str:
    """sha256 of the kernel extension the process would load ("" when it is not built)."""
    from .. import _ext

    path = _ext.so_path()
    if not path or not os.path.exists(path):
        return ""
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


def step_digest(fields: dict) -> str:
    return hashlib.sha256(json.dumps(fields, sort_keys=True, default=str).encode()).hexdigest()[:32]


def identity(cfg, engine: str = "", checkpoint_digest: str = "", guarantee: str = "exact"):
    """The identity of a process serving `cfg` (an EngineConfig)."""
    commit, dirty = _repo_commit()
    m = cfg.model
    step = {"dtype": str(cfg.dtype), "block_size": cfg.block_size, "max_batch": cfg.max_batch,
            "max_model_len": cfg.max_model_len, "graphs": cfg.use_cuda_graphs, "kernels": extension_digest()}
    nccl = ".".join(map(str, torch.cuda.nccl.version())) if torch.cuda.is_available() else ""
    return sp.SoftwareIdentity(
        engine=engine, engine_commit=commit, adapter_commit=commit, adapter_dirty=dirty,
        torch_version=torch.__version__, cuda_version=str(torch.version.cuda or ""), nccl_version=nccl,
        model=m.name, checkpoint_digest=checkpoint_digest or f"random-init:seed{cfg.seed}",
        model_dtype=str(cfg.dtype).replace("torch.", ""),
        kv_format=sp.KvFormat(dtype=str(cfg.dtype).replace("torch.", ""), block_size=cfg.block_size,
                              layout_hash="heads_blocked"),
        layout=sp.ParallelLayout(tensor=cfg.tensor_parallel, pipeline=cfg.pipeline_parallel, data=1, expert=1,
                                 context=1),
        step=sp.StepConfig(digest=step_digest(step), fields={k: str(v) for k, v in step.items()}),
        guarantee=guarantee, serves_changes=True)


def mismatch(a, b) -> list[str]:
    """Fields that differ between two identities and matter for exact replay."""
    out = []
    for f in _EXACT_FIELDS:
        va, vb = getattr(a, f), getattr(b, f)
        if hasattr(va, "SerializeToString"):
            same = va.SerializeToString(deterministic=True) == vb.SerializeToString(deterministic=True)
        else:
            same = va == vb
        if not same:
            out.append(f)
    return out
