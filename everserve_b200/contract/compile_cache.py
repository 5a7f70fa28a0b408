"""A rank's compile cache: the built kernel artifacts it loads, moved between nodes by the stores.

This framework compiles ahead of time (no tracing compiler), so what a rank "compiled" is the
sm_100a kernel extension it loads. A serving worker publishes it into its node store's cache
directory and registers the pair (``CompileCache``: key, digest):

* the key names what the artifact is compatible with: this framework, torch and CUDA versions,
  the target architecture and a digest of the kernel sources;
* the digest names the bytes: sha256 over the manifest's (path, sha256) lines.

Layout: ``<dir>/<key>/<digest>/manifest.json`` and ``<dir>/<key>/<digest>/files/<path>``; the
manifest is written last, so a manifest present is the whole set in place. A spare on a node
whose extension is missing asks its daemon (``CacheWanted``); the daemon has its store fetch the
rank's set from the stores of the nodes that placed it (``CacheFetch``: per-file sha256, chunked
reads), answers ``CacheReady``, and the spare loads the extension from there
(``ES_EXTENSION_PATH``). A spare never builds for itself: one whose set cannot be placed on its
node is refused (``CacheRefused``).

Reference parity: core/everserve/contract/compile_cache.py:37-318 (key, digest, per-rank
manifests) and controller/src/node/cache.rs (the daemon's fetch through the node's store).
"""

from __future__ import annotations

import glob
import hashlib
import json
import os
import shutil
import time

from ..proto import signals as sp

_PKG = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _sha256_file(path: str) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


def source_digest() -> str:
    """sha256 over the kernel sources (file names and bytes, in name order)."""
    h = hashlib.sha256()
    for path in sorted(glob.glob(os.path.join(_PKG, "csrc", "*"))):
        if os.path.isfile(path):
            h.update(os.path.basename(path).encode() + b"\0")
            with open(path, "rb") as f:
                h.update(f.read())
    return h.hexdigest()


def cache_key() -> str:
    import torch

    spec = {"framework": "everserve_b200", "torch": torch.__version__, "cuda": torch.version.cuda or "",
            "arch": "sm_100a", "sources": source_digest()}
    return "es-" + hashlib.sha256(json.dumps(spec, sort_keys=True).encode()).hexdigest()[:32]


def artifacts() -> list[str]:
    """The built files a rank loads: the kernel extension."""
    return sorted(glob.glob(os.path.join(_PKG, "_C*.so")))


def manifest_of(files: dict[str, str]) -> tuple[str, list[dict]]:
    """(digest, manifest entries) of {relative path: file}."""
    entries = [{"path": rel, "size": os.path.getsize(p), "sha256": _sha256_file(p)} for rel, p in sorted(files.items())]
    h = hashlib.sha256()
    for e in entries:
        h.update(f"{e['path']}\0{e['sha256']}\n".encode())
    return h.hexdigest(), entries


def publish(cache_dir: str, files: list[str] | None = None, key: str | None = None):
    """Place this process's artifacts (or `files`) in `cache_dir`; returns the ``CompileCache``
    pair, or None when there is nothing built to publish."""
    files = artifacts() if files is None else files
    if not files:
        return None
    key = key or cache_key()
    digest, entries = manifest_of({os.path.basename(f): f for f in files})
    base = os.path.join(cache_dir, key, digest)
    man = os.path.join(base, "manifest.json")
    if not os.path.exists(man):
        os.makedirs(os.path.join(base, "files"), exist_ok=True)
        for f in files:
            dest = os.path.join(base, "files", os.path.basename(f))
            tmp = dest + f".part{os.getpid()}"
            shutil.copyfile(f, tmp)
            os.replace(tmp, dest)
        tmp = man + f".part{os.getpid()}"
        with open(tmp, "w") as fh:
            json.dump({"key": key, "digest": digest, "files": entries}, fh)
        os.replace(tmp, man)  # last: the set is in place
    return sp.CompileCache(key=key, digest=digest)


def locate(cache_dir: str, key: str, digest: str) -> dict[str, str]:
    """{relative path: file} of a set in place (empty when it is not)."""
    base = os.path.join(cache_dir, key, digest)
    try:
        with open(os.path.join(base, "manifest.json")) as fh:
            man = json.load(fh)
    except (OSError, ValueError):
        return {}
    if man.get("key") != key or man.get("digest") != digest:
        return {}
    return {e["path"]: os.path.join(base, "files", e["path"]) for e in man.get("files", [])}


class CacheRefused(RuntimeError):
    pass


def want(daemon: str, engine: str, rank: int, timeout_s: float = 600.0):
    """Ask this node's daemon for `rank`'s set; returns the ``CacheReady`` once it is in the node's
    store, or raises ``CacheRefused`` with the daemon's reason."""
    from .daemon import _Link

    link = _Link(daemon, timeout_s=10.0)
    try:
        link.send(sp.Signal(cache_wanted=sp.CacheWanted(engine=engine, rank=rank)))
        deadline = time.monotonic() + timeout_s
        while time.monotonic() < deadline:
            link.sock.settimeout(max(0.1, deadline - time.monotonic()))
            try:
                sig = link.recv()
            except TimeoutError:
                break
            kind = sig.WhichOneof("kind")
            if kind == "cache_ready" and sig.cache_ready.engine == engine:
                return sig.cache_ready
            if kind == "cache_refused" and sig.cache_refused.engine == engine:
                raise CacheRefused(sig.cache_refused.reason)
        raise CacheRefused(f"no answer within {timeout_s} s")
    finally:
        link.close()


def load_from_cache(cache_dir: str, ready) -> str:
    """Point the extension loader at the fetched set's extension; returns its path."""
    files = locate(cache_dir, ready.key, ready.digest)
    so = [p for rel, p in files.items() if rel.startswith("_C") and rel.endswith(".so")]
    if not so:
        raise CacheRefused(f"the set {ready.key}/{ready.digest} holds no kernel extension")
    os.environ["ES_EXTENSION_PATH"] = so[0]
    return so[0]
