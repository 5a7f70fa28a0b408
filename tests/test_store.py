"""The C++ KV store (everserve-store) through the Python mirror client and MirrorCommittedKV."""

import time

import pytest
import torch

from cpp_bins import Proc, binary, free_port, wait_socket
from everserve_b200.proto import mirror as pb
from everserve_b200.state.kvcopy import PagedKV
from everserve_b200.state.mirror import MirrorClient, MirrorCommittedKV, MirrorError


@pytest.fixture
def store(tmp_path):
    sock = f"unix:{tmp_path}/store.sock"
    p = Proc([binary("everserve-store"), "--socket", sock, "--data-dir", str(tmp_path / "data"), "--slots", "4096",
              "--budget-bytes", str(1 << 30)])
    wait_socket(sock)
    yield sock
    p.stop()


def _caches(layers=3, nb=32, H=2, bs=16, d=64, seed=0):
    g = torch.Generator().manual_seed(seed)
    kv = PagedKV("heads_blocked", nb, bs, H, d)
    return [torch.randn(kv.shape(), generator=g) for _ in range(layers)], kv


def test_commit_restore_roundtrip(store):
    caches, kv = _caches()
    ckv = MirrorCommittedKV(MirrorClient(store), "eng", 1, caches, kv, store_slots=4096)
    ckv.commit(epoch=1, step=1, counts={"a": 5, "b": 3}, slots=list(range(0, 5)) + [16, 17, 18])
    ckv.commit(epoch=1, step=2, counts={"a": 6, "b": 4}, slots=[5, 19, -1])
    ckv.fence(2)
    spare_caches = [torch.zeros_like(c) for c in caches]
    spare = MirrorCommittedKV(MirrorClient(store), "eng", 7, spare_caches, kv)
    counts = spare.restore(1)
    assert counts == {"a": 6, "b": 4}
    heads = torch.arange(kv.heads)
    written = torch.tensor([0, 1, 2, 3, 4, 5, 16, 17, 18, 19])
    for c, s in zip(caches, spare_caches):
        assert torch.equal(kv.rows_of_heads(s, written, heads), kv.rows_of_heads(c, written, heads))
    # an untouched slot stays empty on the spare
    assert torch.count_nonzero(kv.rows_of_heads(spare_caches[0], torch.tensor([40]), heads)) == 0
    # only what was written since step 1
    since = MirrorClient(store).restore("eng", 1, since_step=1)
    slots = {s for t in since.tables for r in t.written for s in range(r.start, r.start + r.count)}
    assert slots == {5, 19}
    ckv.close()
    spare.close()


def test_stale_epoch_refused_and_counts(store):
    caches, kv = _caches(layers=1)
    c = MirrorClient(store)
    ckv = MirrorCommittedKV(c, "e2", 0, caches, kv)
    ckv.commit(epoch=3, step=10, counts={"r": 9}, slots=[1, 2])
    ckv.fence(10)
    with pytest.raises(MirrorError, match="stale epoch"):
        c.commit("e2", 0, 2, 11, None, {"r": 10})
    assert c.committed("e2", ["r", "nope"]) == {"r": 9, "nope": 0}
    ckv.evicted("r", 4)
    assert c.committed("e2", ["r"]) == {"r": 4}
    ckv.finished("r")
    assert c.committed("e2", ["r"]) == {"r": 0}
    ckv.close()


def test_replication_between_stores(tmp_path):
    port = free_port()
    sock_a, sock_b = f"unix:{tmp_path}/a.sock", f"unix:{tmp_path}/b.sock"
    a = Proc([binary("everserve-store"), "--socket", sock_a, "--data-dir", str(tmp_path / "a"), "--slots", "1024"])
    b = Proc([binary("everserve-store"), "--socket", sock_b, "--data-dir", str(tmp_path / "b"), "--slots", "1024",
              "--replica-listen", f"127.0.0.1:{port}"])
    try:
        wait_socket(sock_a)
        wait_socket(sock_b)
        wait_socket(f"127.0.0.1:{port}")
        caches, kv = _caches(layers=2)
        ca = MirrorClient(sock_a)
        ckv = MirrorCommittedKV(ca, "rep", 2, caches, kv)
        ca.replicate("rep", 2, [f"127.0.0.1:{port}"])
        ckv.commit(epoch=1, step=1, counts={"x": 3}, slots=[0, 1, 2])
        ckv.fence(1)
        cb = MirrorClient(sock_b)
        deadline = time.monotonic() + 5
        while time.monotonic() < deadline and cb.committed("rep", ["x"])["x"] != 3:
            time.sleep(0.02)
        assert cb.committed("rep", ["x"]) == {"x": 3}
        spare_caches = [torch.zeros_like(c) for c in caches]
        spare = MirrorCommittedKV(cb, "rep", 5, spare_caches, kv)
        assert spare.restore(2) == {"x": 3}
        heads = torch.arange(kv.heads)
        for c, s in zip(caches, spare_caches):
            assert torch.equal(kv.rows_of_heads(s, torch.tensor([0, 1, 2]), heads),
                               kv.rows_of_heads(c, torch.tensor([0, 1, 2]), heads))
        # a replicated part whose checksum does not match is refused whole
        bad = pb.Replicated(engine="rep", rank=9, epoch=1, step=1, tables=[pb.ReplicatedTable(
            table=0, dtype="float32", shape=[2, 64], slots=[3], data=b"\0" * 512, crc32c=[12345])])
        with pytest.raises(MirrorError, match="checksum"):
            cb.call(pb.MirrorRequest(replicated=bad))
        ckv.close()
        spare.close()
    finally:
        a.stop()
        b.stop()
