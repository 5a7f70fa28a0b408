"""Wire compatibility of the control plane's generated C++ codec with google.protobuf.

Every message of the six schemas is filled field by field (scalars at their edges: negative int32
in ten-byte varints, uint64 and fixed64 maxima, NaN-free floats, unicode strings, bytes; enums;
nested messages; repeated fields with several elements; maps; oneof members; proto3 ``optional``
fields set to their zero value, whose presence must survive) and encoded by google.protobuf from
the same schemas. The C++ codec (``everserve-codec-check``) decodes and re-encodes the bytes; the
result must parse back to the same message. The same holds with unknown fields of every wire type
appended (they are skipped), and with repeated scalars sent unpacked (proto3 packs them, decoders
must accept both). The coordinator's policy reader takes google.protobuf's proto3 JSON of a Policy.

Reference parity: core/tests/test_wire.py, test_signals.py and test_signals_coverage.py check the
same schemas' encodings between the reference's Python and Rust sides.
"""

import random
import struct
import subprocess

import pytest
from google.protobuf import descriptor as d
from google.protobuf import json_format

from everserve_b200.proto import CLASSES, policy as pp, signals as sp

import cpp_bins

FD = d.FieldDescriptor


def _repeated(f) -> bool:
    return f.is_repeated if hasattr(f, "is_repeated") else f.label == FD.LABEL_REPEATED


def _check_bin():
    return cpp_bins.binary("everserve-codec-check")


def _run(lines: list[str]) -> list[str]:
    out = subprocess.run([_check_bin()], input="\n".join(lines) + "\n", capture_output=True, text=True, timeout=120,
                         check=True).stdout
    return out.splitlines()


def _scalar(f, rnd: random.Random, zero: bool = False):
    t = f.type
    if t in (FD.TYPE_INT32, FD.TYPE_SINT32, FD.TYPE_SFIXED32):
        return 0 if zero else rnd.choice([-1, -(2 ** 31), 2 ** 31 - 1, 7, -300])
    if t in (FD.TYPE_INT64, FD.TYPE_SINT64, FD.TYPE_SFIXED64):
        return 0 if zero else rnd.choice([-1, -(2 ** 63), 2 ** 63 - 1, 1 << 40, -5])
    if t in (FD.TYPE_UINT32, FD.TYPE_FIXED32):
        return 0 if zero else rnd.choice([1, 2 ** 32 - 1, 128, 300])
    if t in (FD.TYPE_UINT64, FD.TYPE_FIXED64):
        return 0 if zero else rnd.choice([1, 2 ** 64 - 1, 1 << 35, 16384])
    if t == FD.TYPE_BOOL:
        return not zero
    if t == FD.TYPE_FLOAT:
        return 0.0 if zero else rnd.choice([1.5, -0.25, 3.0e38, 1e-30])
    if t == FD.TYPE_DOUBLE:
        return 0.0 if zero else rnd.choice([1.5, -2.5e300, 1e-300, 0.1])
    if t == FD.TYPE_STRING:
        return "" if zero else rnd.choice(["a", "rank-7", "nœud/ü", "x" * 200])
    if t == FD.TYPE_BYTES:
        return b"" if zero else bytes(rnd.randrange(256) for _ in range(rnd.choice([1, 3, 130])))
    if t == FD.TYPE_ENUM:
        vals = [v.number for v in f.enum_type.values]
        return vals[0] if zero else rnd.choice([v for v in vals if v != 0] or vals)
    raise TypeError(t)


def _synthetic(o) -> bool:
    """The oneof proto3 makes for an ``optional`` field (one field, named after it)."""
    return len(o.fields) == 1 and o.name == "_" + o.fields[0].name


def _fill(msg, rnd: random.Random, depth: int = 0) -> None:
    """Set every field: one member of each oneof, proto3 optional fields to their zero value."""
    oneofs_done = set()
    for f in msg.DESCRIPTOR.fields:
        o = f.containing_oneof
        optional = o is not None and _synthetic(o)
        if o is not None and not optional:
            if o.name in oneofs_done:
                continue
            oneofs_done.add(o.name)
        is_map = f.message_type is not None and f.message_type.GetOptions().map_entry
        if is_map:
            kf, vf = f.message_type.fields_by_name["key"], f.message_type.fields_by_name["value"]
            m = getattr(msg, f.name)
            for _ in range(2):
                k = _scalar(kf, rnd)
                if vf.type == FD.TYPE_MESSAGE:
                    if depth < 3:
                        _fill(m[k], rnd, depth + 1)
                else:
                    m[k] = _scalar(vf, rnd)
            continue
        if _repeated(f):
            rep = getattr(msg, f.name)
            for _ in range(3):
                if f.type == FD.TYPE_MESSAGE:
                    if depth < 3:
                        _fill(rep.add(), rnd, depth + 1)
                else:
                    rep.append(_scalar(f, rnd))
            continue
        if f.type == FD.TYPE_MESSAGE:
            if depth < 3:
                sub = getattr(msg, f.name)
                sub.SetInParent()
                _fill(sub, rnd, depth + 1)
            continue
        setattr(msg, f.name, _scalar(f, rnd, zero=optional))


def _messages():
    return sorted((n, c) for n, c in CLASSES.items() if not c.DESCRIPTOR.GetOptions().map_entry)


def test_every_message_round_trips_through_the_cpp_codec():
    rnd = random.Random(0)
    cases = []
    for name, cls in _messages():
        for _ in range(2):
            m = cls()
            _fill(m, rnd)
            cases.append((name, cls, m))
    assert len(cases) >= 2 * 100
    got = _run([f"{n} {m.SerializeToString().hex()}" for n, _, m in cases])
    bad = []
    for (name, cls, m), line in zip(cases, got):
        if line == "ERR":
            bad.append(f"{name}: refused")
            continue
        back = cls()
        back.ParseFromString(bytes.fromhex(line))
        if back != m:
            bad.append(f"{name}: {m} != {back}")
    assert not bad, bad[:5]


def _varint(v: int) -> bytes:
    v &= (1 << 64) - 1
    out = bytearray()
    while True:
        b = v & 0x7F
        v >>= 7
        if v:
            out.append(b | 0x80)
        else:
            out.append(b)
            return bytes(out)


def test_unknown_fields_of_every_wire_type_are_skipped():
    rnd = random.Random(1)
    unknown = (_varint((5000 << 3) | 0) + _varint(2 ** 63)            # varint
               + _varint((5001 << 3) | 1) + struct.pack("<d", 1.5)    # fixed64
               + _varint((5002 << 3) | 2) + _varint(4) + b"abcd"      # length-delimited
               + _varint((5003 << 3) | 5) + struct.pack("<I", 7))     # fixed32
    cases = []
    for name, cls in _messages():
        m = cls()
        _fill(m, rnd)
        cases.append((name, cls, m))
    got = _run([f"{n} {(unknown + m.SerializeToString() + unknown).hex()}" for n, _, m in cases])
    for (name, cls, m), line in zip(cases, got):
        assert line != "ERR", name
        back = cls()
        back.ParseFromString(bytes.fromhex(line))
        assert back == m, name


def _unpacked(msg) -> bytes:
    """The message's encoding with every repeated scalar field written element by element."""
    out = bytearray()
    rest = type(msg)()
    rest.CopyFrom(msg)
    for f in msg.DESCRIPTOR.fields:
        if not _repeated(f) or f.type in (FD.TYPE_MESSAGE, FD.TYPE_STRING, FD.TYPE_BYTES):
            continue
        for v in getattr(msg, f.name):
            if f.type in (FD.TYPE_FIXED64, FD.TYPE_SFIXED64, FD.TYPE_DOUBLE):
                fmt = {FD.TYPE_FIXED64: "<Q", FD.TYPE_SFIXED64: "<q", FD.TYPE_DOUBLE: "<d"}[f.type]
                out += _varint((f.number << 3) | 1) + struct.pack(fmt, v)
            elif f.type in (FD.TYPE_FIXED32, FD.TYPE_SFIXED32, FD.TYPE_FLOAT):
                fmt = {FD.TYPE_FIXED32: "<I", FD.TYPE_SFIXED32: "<i", FD.TYPE_FLOAT: "<f"}[f.type]
                out += _varint((f.number << 3) | 5) + struct.pack(fmt, v)
            elif f.type in (FD.TYPE_SINT32, FD.TYPE_SINT64):
                zz = (v << 1) ^ (v >> 63)
                out += _varint((f.number << 3) | 0) + _varint(zz)
            else:
                out += _varint((f.number << 3) | 0) + _varint(int(v))
        rest.ClearField(f.name)
    return bytes(out) + rest.SerializeToString()


def test_repeated_scalars_sent_unpacked_are_accepted():
    rnd = random.Random(2)
    cases = []
    for name, cls in _messages():
        if not any(_repeated(f) and f.type not in (FD.TYPE_MESSAGE, FD.TYPE_STRING, FD.TYPE_BYTES)
                   for f in cls.DESCRIPTOR.fields):
            continue
        m = cls()
        _fill(m, rnd)
        data = _unpacked(m)
        check = cls()
        check.ParseFromString(data)
        assert check == m  # the hand encoding is a valid one
        cases.append((name, cls, m, data))
    assert cases
    got = _run([f"{n} {data.hex()}" for n, _, _, data in cases])
    for (name, cls, m, _), line in zip(cases, got):
        assert line != "ERR", name
        back = cls()
        back.ParseFromString(bytes.fromhex(line))
        assert back == m, name


def test_truncated_messages_are_refused():
    rnd = random.Random(3)
    lines, names = [], []
    for name, cls in _messages():
        m = cls()
        _fill(m, rnd)
        data = m.SerializeToString()
        if len(data) < 4:
            continue
        names.append(name)
        lines.append(f"{name} {data[:-1].hex()}")  # the last field cut short
    got = _run(lines)
    refused = sum(1 for line in got if line == "ERR")
    # cutting the last byte breaks a length, a varint or a fixed-width value: refused unless the last
    # field happened to be a one-byte-shorter valid encoding (a varint's continuation is never that)
    assert refused >= 0.9 * len(lines), (refused, len(lines))


@pytest.mark.parametrize("names", [False, True])
def test_policy_json_from_google_protobuf(names):
    pol = pp.Policy(outcomes_in_order=[sp.OUTCOME_REPLACE, sp.OUTCOME_SHRINK], max_concurrent_losses=2)
    e = pol.engines.add(name="e0", tensor_parallel=4, pipeline_parallel=2, data_parallel=1,
                        placement_independent_model=True)
    e.spares.add(node="n1", device=4, rank=2)
    pol.engines.add(name="e1", tensor_parallel=8)
    text = json_format.MessageToJson(pol, preserving_proto_field_name=names)
    (line,) = _run([f"policy {text.encode().hex()}"])
    assert not line.startswith("ERR"), line
    import json

    got = json.loads(line)
    assert got["outcomes"] == [sp.OUTCOME_REPLACE, sp.OUTCOME_SHRINK]
    assert got["maxConcurrentLosses"] == 2
    assert got["engines"]["e0"] == {"tp": 4, "pp": 2, "dp": 1, "placementIndependent": True}
    assert got["engines"]["e1"]["tp"] == 8 and got["engines"]["e1"]["pp"] == 1
