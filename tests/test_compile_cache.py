"""Compile caches moved between nodes by their stores, through the real binaries.

A worker on n0 publishes its build into n0's cache and registers the pair; the coordinator
places it with n0's store as holder. A process on n1 asks its daemon for the rank's set: n1's
store fetches it from n0's store chunk by chunk, checks every file's sha256, and the daemon
answers CacheReady; the loader then takes the fetched file. A rank with no pair placed is
refused, and so is a set whose holder's bytes no longer match its manifest.
"""

import hashlib
import os

import pytest

from everserve_b200.contract import compile_cache as cc
from everserve_b200.contract.daemon import DaemonConnection
from everserve_b200.serving.cluster import ControlPlane

from test_control_cpu import _P, _wait


def _artifact(path, n):
    data = hashlib.sha256(b"seed").digest() * (n // 32 + 1)
    with open(path, "wb") as f:
        f.write(data[:n])
    return str(path)


def test_publish_digest_is_content_addressed(tmp_path):
    a = _artifact(tmp_path / "_C.test.so", 1000)
    p1 = cc.publish(str(tmp_path / "cache"), [a], key="k1")
    p2 = cc.publish(str(tmp_path / "cache"), [a], key="k1")
    assert p1.digest == p2.digest and p1.key == "k1"
    files = cc.locate(str(tmp_path / "cache"), "k1", p1.digest)
    assert list(files) == ["_C.test.so"] and open(files["_C.test.so"], "rb").read() == open(a, "rb").read()
    with open(a, "ab") as f:
        f.write(b"x")
    assert cc.publish(str(tmp_path / "cache"), [a], key="k1").digest != p1.digest
    assert cc.locate(str(tmp_path / "cache"), "k1", "0" * 64) == {}
    assert cc.cache_key().startswith("es-")


def test_spare_node_fetches_the_ranks_build_from_the_holder(tmp_path):
    with ControlPlane(str(tmp_path / "cp"), engines=[{"name": "e0", "tensorParallel": 2}], extra_nodes=["n1"],
                      node_args=["--cache-wait-ms", "3000"]) as cp:
        # 9 MiB + change: three chunks of at most 4 MiB each
        art = _artifact(tmp_path / "_C.cpython-312-x86_64-linux-gnu.so", 9 * (1 << 20) + 123)
        pair = cc.publish(cp.cache_dirs["n0"], [art], key="es-test")
        w0 = DaemonConnection(cp.daemon_sockets["n0"], "e0", _P(0), node="n0", compile_cache=pair)
        assert _wait(lambda: cp.engine_view("e0")["status"]["workers"])
        # a spare starting on n1 first asks for the engine's start-up record (the coordinator then
        # sends n1 the engine's placement), then for its rank's build
        from everserve_b200.contract.daemon import _Link
        from everserve_b200.proto import signals as sp

        ask = _Link(cp.daemon_sockets["n1"])
        ask.send(sp.Signal(replay_ask=sp.ReplayAsk(engine="e0", rank=0)))
        ready = cc.want(cp.daemon_sockets["n1"], "e0", 0, timeout_s=30)
        ask.close()
        assert (ready.key, ready.digest) == (pair.key, pair.digest)
        got = cc.locate(cp.cache_dirs["n1"], pair.key, pair.digest)
        assert open(got[os.path.basename(art)], "rb").read() == open(art, "rb").read()
        # asked again: already in place
        assert cc.want(cp.daemon_sockets["n1"], "e0", 0, timeout_s=30).digest == pair.digest
        path = cc.load_from_cache(cp.cache_dirs["n1"], ready)
        assert os.environ.pop("ES_EXTENSION_PATH") == path
        # rank 1 placed no pair: refused once the daemon's wait runs out
        with pytest.raises(cc.CacheRefused, match="no compile-cache pair"):
            cc.want(cp.daemon_sockets["n1"], "e0", 1, timeout_s=30)

        # a holder whose bytes no longer match its manifest serves nothing
        bad = _artifact(tmp_path / "_C.other.so", 5000)
        pair2 = cc.publish(cp.cache_dirs["n0"], [bad], key="es-test2")
        target = cc.locate(cp.cache_dirs["n0"], pair2.key, pair2.digest)["_C.other.so"]
        with open(target, "r+b") as f:
            f.write(b"corrupt")
        w1 = DaemonConnection(cp.daemon_sockets["n0"], "e0", _P(1), node="n0", compile_cache=pair2)
        assert _wait(lambda: len(cp.engine_view("e0")["status"]["workers"]) == 2)
        with pytest.raises(cc.CacheRefused, match="sha256"):
            cc.want(cp.daemon_sockets["n1"], "e0", 1, timeout_s=30)
        assert cc.locate(cp.cache_dirs["n1"], pair2.key, pair2.digest) == {}
        for c in (w0, w1):
            c.close()
