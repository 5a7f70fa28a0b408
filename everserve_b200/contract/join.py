"""The two halves of a join, as bytes the control plane carries unread.

When a spare takes a rank, the head offers it the place to link (``Offer``: rank, epoch, the
head's carrier address, a one-time token, whether the rank died or left on a notice) and the spare
answers (``Answer``: what it restored). The daemons and the coordinator relay the bytes without
reading them. The payload is self-describing so a process of another build fails with a named
error instead of misreading it::

    b"everserve-b200-join" 0x00 b"<version>" 0x00 b"<kind>" 0x00 <JSON body>

The body is data only: every field is declared below and checked on the way in (an unknown or a
missing field is refused by name). Nothing in a payload can run as code in the reader.

Reference parity: the tag + version + kind + JSON framing of
adapters/vllm/everserve_vllm/join.py:1-225 (same idea and checks; this framework's fields).
"""

from __future__ import annotations

import dataclasses
import json
from dataclasses import dataclass, field

TAG = b"everserve-b200-join"
VERSION = 1


class JoinFormatError(ValueError):
    pass


@dataclass(frozen=True)
class Offer:
    rank: int
    epoch: int
    carrier: str  # host:port of the head's carrier listener
    token: str  # the carrier hello must present it
    faulted: bool = True  # the rank died (no catch-up needed) rather than left on a notice


@dataclass(frozen=True)
class Answer:
    rank: int
    epoch: int
    restored_step: int = -1
    computed: dict = field(default_factory=dict)
    error: str = ""


_KINDS = {b"offer": Offer, b"answer": Answer}
_TYPES = {int: int, str: str, bool: bool, dict: dict}


def encode(msg: Offer | Answer) -> bytes:
    kind = next(k for k, c in _KINDS.items() if isinstance(msg, c))
    body = json.dumps(dataclasses.asdict(msg), sort_keys=True).encode()
    return b"%s\x00%d\x00%s\x00" % (TAG, VERSION, kind) + body


def decode(payload: bytes) -> Offer | Answer:
    parts = payload.split(b"\x00", 3)
    if len(parts) != 4:
        raise JoinFormatError("not a join payload")
    tag, version, kind, body = parts
    if tag != TAG:
        raise JoinFormatError(f"payload tagged {tag!r}, not {TAG!r}")
    if version != str(VERSION).encode():
        raise JoinFormatError(f"join payload version {version!r}; this build reads {VERSION}")
    cls = _KINDS.get(kind)
    if cls is None:
        raise JoinFormatError(f"unknown join kind {kind!r}")
    try:
        data = json.loads(body)
    except ValueError as e:
        raise JoinFormatError(f"join body is not JSON: {e}") from None
    if not isinstance(data, dict):
        raise JoinFormatError("join body is not an object")
    fields = {f.name: f for f in dataclasses.fields(cls)}
    unknown = set(data) - set(fields)
    if unknown:
        raise JoinFormatError(f"unknown field(s) {sorted(unknown)} in a {kind.decode()}")
    out = {}
    for name, f in fields.items():
        if name not in data:
            if f.default is dataclasses.MISSING and f.default_factory is dataclasses.MISSING:
                raise JoinFormatError(f"missing field {name!r} in a {kind.decode()}")
            continue
        want = f.type if isinstance(f.type, type) else {"int": int, "str": str, "bool": bool, "dict": dict}[f.type]
        v = data[name]
        if want is int and isinstance(v, bool) or not isinstance(v, want):
            raise JoinFormatError(f"field {name!r} is {type(v).__name__}, not {want.__name__}")
        out[name] = v
    return cls(**out)
