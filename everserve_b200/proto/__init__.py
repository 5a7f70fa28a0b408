"""Message classes of the control-plane schemas (proto/everserve/proto/*.proto).

The classes are built at import time from the schemas by :mod:`everserve_b200.proto.protogen`
(the environment has no protoc), in a private descriptor pool. Each schema file is a namespace::

    from everserve_b200.proto import signals, mirror, coord, policy, spec, discovery
    sig = signals.Signal(change=signals.Change(epoch=3, lost=[1]))
    data = sig.SerializeToString()
"""

from __future__ import annotations

import types

from .protogen import build_python, load_all

_FILES = load_all()
POOL, CLASSES = build_python(_FILES)


def _namespace(pkg: str) -> types.SimpleNamespace:
    ns = types.SimpleNamespace()
    for full, cls in CLASSES.items():
        if full.startswith(pkg + "."):
            setattr(ns, full[len(pkg) + 1 :], cls)
    for pf in _FILES.values():
        if pf.package != pkg:
            continue
        for e in pf.enums:
            ed = POOL.FindEnumTypeByName(e.full)
            for v in ed.values:
                setattr(ns, v.name, v.number)
            setattr(ns, e.name, ed)
        for m in pf.messages:
            for e in m.enums:
                ed = POOL.FindEnumTypeByName(e.full)
                for v in ed.values:
                    setattr(getattr(ns, m.name), v.name, v.number)
    return ns


signals = _namespace("everserve.signals.v1")
mirror = _namespace("everserve.mirror.v1")
coord = _namespace("everserve.coord.v1")
policy = _namespace("everserve.policy.v1")
spec = _namespace("everserve.spec.v1")
discovery = _namespace("everserve.discovery.v1")

__all__ = ["signals", "mirror", "coord", "policy", "spec", "discovery", "POOL", "CLASSES"]
