"""The KV store's request protocol, message by message (everserve-store over its Unix socket).

Each test speaks the protobuf messages of `proto/everserve/proto/mirror.proto` directly, the way a
rank, a spare or a peer store does, and checks the store's answer: refusals with their reasons
(names, dtypes, shapes, budget, slots, staging files, stale epochs, checksums), what a commit
leaves behind (rows, their checksums and step stamps, counts), what a restore returns per rank and
since a step, how counts follow evictions and finished requests, and the replica handshake.
Reference parity: the store service behaviours of store/src (tested in store/tests/service.rs).
"""

import os
import struct

import pytest

from cpp_bins import Proc, binary, wait_socket
from everserve_b200.proto import mirror as pb
from everserve_b200.proto import signals as spb
from everserve_b200.state.mirror import MirrorClient, MirrorError

SLOTS = 256


def _crc32c_table():
    table = []
    for i in range(256):
        c = i
        for _ in range(8):
            c = (c >> 1) ^ 0x82F63B78 if c & 1 else c >> 1
        table.append(c)
    return table


_CRC = _crc32c_table()


def crc32c(data: bytes) -> int:
    """CRC-32C (Castagnoli, reflected polynomial 0x82F63B78), bytewise."""
    c = 0xFFFFFFFF
    for b in data:
        c = _CRC[(c ^ b) & 0xFF] ^ (c >> 8)
    return c ^ 0xFFFFFFFF


def test_crc32c_check_value():
    # the published check value of CRC-32C over "123456789"
    assert crc32c(b"123456789") == 0xE3069283


def _start(tmp_path, name="s", budget=1 << 30):
    sock = f"unix:{tmp_path}/{name}.sock"
    p = Proc([binary("everserve-store"), "--socket", sock, "--data-dir", str(tmp_path / name), "--slots", str(SLOTS),
              "--budget-bytes", str(budget)])
    wait_socket(sock)
    return p, sock


@pytest.fixture
def store(tmp_path):
    p, sock = _start(tmp_path)
    yield sock
    p.stop()


def _open(c: MirrorClient, engine: str, rank: int):
    return c.call(pb.MirrorRequest(open=pb.Open(engine=engine, rank=rank, protocol=spb.PROTOCOL_VERSION,
                                                protocol_oldest=spb.PROTOCOL_OLDEST))).opened


# one table row: [2 (k, v), 4] float32 = 32 bytes
SHAPE = [2, 4]
ROW = 2 * 4 * 4


def _stage(c: MirrorClient, engine: str, rank: int, rows: list[bytes], tag: str = "a") -> str:
    """Write `rows` (one layer, one head) into a staging file in the rank's directory."""
    o = _open(c, engine, rank)
    name = o.stage_prefix + tag
    with open(os.path.join(o.rank_dir, name), "wb") as f:
        f.write(b"".join(rows))
    return name


def _row(v: float) -> bytes:
    return struct.pack("<8f", *[v + i for i in range(8)])


def _commit(c, engine, rank, epoch, step, stage, slots, counts=None, layers=(0,), heads=(0,)):
    counts = counts or {}
    staged = pb.StagedStep(stage=stage, base_offset=0, layer_stride=len(slots) * ROW * len(heads),
                           head_stride=len(slots) * ROW, layers=list(layers), heads=list(heads), table_stride=1000,
                           slots=list(slots), dtype="float32", shape=SHAPE)
    return c.commit(engine, rank, epoch, step, staged, counts)


def test_refusals_name_their_reason(tmp_path):
    p, sock = _start(tmp_path, budget=64 * 1024)
    c = MirrorClient(sock)
    try:
        with pytest.raises(MirrorError, match="bad engine name"):
            _open(c, "../up", 0)
        with pytest.raises(MirrorError, match="unknown dtype"):
            c.prepare("e", 0, [0], "int7", SHAPE, SLOTS)
        c.prepare("e", 0, [0], "float32", SHAPE, SLOTS)  # 256 rows of 32 bytes: 8 KB of the budget
        with pytest.raises(MirrorError, match="differs from the table's"):
            c.prepare("e", 0, [0], "float32", [2, 8], SLOTS)
        with pytest.raises(MirrorError, match="budget"):
            c.prepare("e", 0, [1], "float32", [2, 64], SLOTS)  # 128 KB more than the 64 KB budget
        st = _stage(c, "e", 0, [_row(1.0), _row(2.0)])
        with pytest.raises(MirrorError, match="bad stage name"):
            _commit(c, "e", 0, 1, 1, "../" + st, [0, 1])
        with pytest.raises(MirrorError, match="outside the store"):
            _commit(c, "e", 0, 1, 1, st, [0, SLOTS])
        with pytest.raises(MirrorError, match="shorter than the descriptor"):
            _commit(c, "e", 0, 1, 1, st, [0, 1, 2])
        # nothing of a refused commit was applied
        assert c.committed("e", ["r"]) == {"r": 0}
        assert _commit(c, "e", 0, 2, 5, st, [0, 1], {"r": 2}) == 5
        with pytest.raises(MirrorError, match="stale epoch 1"):
            _commit(c, "e", 0, 1, 6, st, [0, 1], {"r": 9})
        assert c.committed("e", ["r"]) == {"r": 2}
        # a later epoch is accepted and moves the rank on
        assert _commit(c, "e", 0, 3, 7, st, [2, 3], {"r": 4}) == 7
        assert c.committed("e", ["r"]) == {"r": 4}
    finally:
        c.close()
        p.stop()


def test_committed_rows_carry_their_step_and_checksum(store):
    c = MirrorClient(store)
    rows = [_row(10.0 * i) for i in range(5)]
    st = _stage(c, "e", 0, rows)
    _commit(c, "e", 0, 1, 0, st, [3, 4, -1, 9, 10])  # -1: a padded row, skipped
    st2 = _stage(c, "e", 0, [_row(-1.0)], tag="b")
    _commit(c, "e", 0, 1, 12, st2, [4])  # rewrites slot 4 at step 12
    rep = c.call(pb.MirrorRequest(rows=pb.RowsQuery(engine="e", rank=0, table=0, slots=[3, 4, 5, 9, 10, SLOTS, -3])))
    got = {r.slot: r for r in rep.rows.rows}
    assert sorted(got) == [3, 4, 5, 9, 10]  # slots outside the store are left out
    assert got[3].data == rows[0] and got[9].data == rows[3] and got[10].data == rows[4]
    assert got[4].data == _row(-1.0)
    assert got[3].written_step == 1  # step 0 is stamped 1: 0 means never written
    assert got[4].written_step == 12
    assert got[5].written_step == 0 and got[5].data == bytes(ROW)
    for s in (3, 4, 9, 10):
        assert got[s].crc32c == crc32c(got[s].data)
    assert rep.rows.epoch == 1 and rep.rows.step == 12
    c.close()


def test_restore_is_per_rank_and_since_a_step(store):
    c = MirrorClient(store)
    st0 = _stage(c, "e", 0, [_row(1.0), _row(2.0), _row(3.0)])
    _commit(c, "e", 0, 1, 4, st0, [0, 1, 2], {"a": 3})
    st0b = _stage(c, "e", 0, [_row(4.0)], tag="b")
    _commit(c, "e", 0, 1, 5, st0b, [7], {"a": 4})
    # layer 1 of the staging file starts one layer stride (two rows) in
    st1 = _stage(c, "e", 1, [bytes(ROW), bytes(ROW), _row(9.0), _row(8.0)], tag="c")
    _commit(c, "e", 1, 1, 5, st1, [20, 21], {"a": 4}, layers=(1,), heads=(0,))

    def written(rep):
        return {t.layer: sorted(s for r in t.written for s in range(r.start, r.start + r.count)) for t in rep.tables}

    r0 = c.restore("e", 0)
    assert written(r0) == {0: [0, 1, 2, 7]}
    assert dict(zip(r0.request_ids, r0.committed_tokens)) == {"a": 4} and r0.step == 5
    assert [list(t.shape) for t in r0.tables] == [[SLOTS] + SHAPE]
    assert written(c.restore("e", 0, since_step=4)) == {0: [7]}
    assert written(c.restore("e", 1)) == {1000: [20, 21]}  # layer 1, head 0: table 1 * 1000 + 0
    assert written(c.restore("e", 2)) == {}  # a rank that never committed
    assert written(c.restore("other", 0)) == {}
    # the restored table file holds the rows at their slots
    path = next(t.path for t in r0.tables)
    with open(path, "rb") as f:
        f.seek(7 * ROW)
        assert f.read(ROW) == _row(4.0)
    c.close()


def test_counts_follow_evictions_and_finished_requests(store):
    c = MirrorClient(store)
    st = _stage(c, "e", 0, [_row(0.0)])
    _commit(c, "e", 0, 1, 1, st, [0], {"a": 10, "b": 7})
    st1 = _stage(c, "e", 1, [_row(0.0)], tag="b")
    _commit(c, "e", 1, 1, 1, st1, [0], {"a": 10, "b": 7})
    assert c.committed("e", ["a", "b", "x"]) == {"a": 10, "b": 7, "x": 0}
    c.evicted("e", "a", 4)  # preempted: only its first 4 tokens' rows stay valid
    assert c.committed("e", ["a"]) == {"a": 4}
    for rank in (0, 1):  # every rank's record follows
        r = c.restore("e", rank)
        assert dict(zip(r.request_ids, r.committed_tokens))["a"] == 4
    c.finished("e", ["b"])
    assert c.committed("e", ["a", "b"]) == {"a": 4, "b": 0}
    assert "b" not in c.restore("e", 1).request_ids
    assert c.committed("unknown-engine", ["a"]) == {"a": 0}
    c.close()


def _replicated(epoch, step, slots, rows, crcs=None, table=0, counts=None):
    counts = counts or {}
    crcs = [crc32c(r) for r in rows] if crcs is None else crcs
    return pb.MirrorRequest(replicated=pb.Replicated(
        engine="e", rank=0, epoch=epoch, step=step,
        tables=[pb.ReplicatedTable(table=table, dtype="float32", shape=SHAPE, slots=list(slots), data=b"".join(rows),
                                   crc32c=list(crcs))],
        request_ids=list(counts), committed_tokens=list(counts.values())))


def test_replicated_parts_are_checked_whole_before_any_write(store):
    """A peer's replicated part: applied when every row's checksum holds; refused whole (nothing
    written, counts untouched) on a bad checksum, a row/checksum count mismatch, a slot outside the
    store or a stale epoch."""
    c = MirrorClient(store)
    good = [_row(1.0), _row(2.0)]
    c.call(_replicated(2, 8, [5, 6], good, counts={"q": 7}))
    assert c.committed("e", ["q"]) == {"q": 7}
    bad = [_row(3.0), _row(4.0)]
    with pytest.raises(MirrorError, match="slot 11: checksum mismatch"):
        c.call(_replicated(2, 9, [10, 11], bad, crcs=[crc32c(bad[0]), 0], counts={"q": 9}))
    with pytest.raises(MirrorError, match="rows and checksums do not match"):
        c.call(_replicated(2, 9, [10, 11], bad, crcs=[crc32c(bad[0])]))
    with pytest.raises(MirrorError, match="slot out of range"):
        c.call(_replicated(2, 9, [10, SLOTS], bad))
    with pytest.raises(MirrorError, match="stale epoch"):
        c.call(_replicated(1, 9, [10, 11], bad))
    assert c.committed("e", ["q"]) == {"q": 7}
    rep = c.call(pb.MirrorRequest(rows=pb.RowsQuery(engine="e", rank=0, table=0, slots=[5, 6, 10, 11])))
    got = {r.slot: (r.data, r.written_step) for r in rep.rows.rows}
    assert got[5] == (good[0], 8) and got[6] == (good[1], 8)
    assert got[10][1] == 0 and got[11][1] == 0  # no part of a refused message landed
    c.close()


def test_replica_state_and_caught_up(store):
    c = MirrorClient(store)

    def state():
        return c.call(pb.MirrorRequest(replica_state=pb.ReplicaStateQuery(
            engine="e", rank=0, protocol=spb.PROTOCOL_VERSION, protocol_oldest=spb.PROTOCOL_OLDEST))).replica_state

    s = state()
    assert (s.epoch, s.step, s.held, s.caught_up) == (0, 0, False, False)
    c.call(_replicated(4, 20, [1], [_row(5.0)]))
    s = state()
    assert (s.epoch, s.step, s.held, s.caught_up) == (4, 20, True, False)
    with pytest.raises(MirrorError, match="stale epoch"):
        c.call(pb.MirrorRequest(caught_up=pb.CaughtUp(engine="e", rank=0, epoch=3, step=20)))
    c.call(pb.MirrorRequest(caught_up=pb.CaughtUp(engine="e", rank=0, epoch=4, step=20)))
    assert state().caught_up
    c.close()
