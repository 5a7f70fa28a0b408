"""A small .proto (proto3) parser and code generator; this environment has no protoc.

It reads the schemas under ``proto/everserve/proto`` and

* builds ``FileDescriptorProto`` objects at import time, so ``everserve_b200.proto`` exposes the
  message classes through the installed ``google.protobuf`` runtime (binary and proto3-JSON codecs
  included);
* emits the C++ header of the control plane (``python -m everserve_b200.proto.protogen --cpp OUT``):
  one struct per message with a hand-written varint / length-delimited encoder and decoder.

The subset covers what the schemas use: packages, imports, enums (top level and nested), messages
(nested enums), scalar / enum / message / repeated / optional / map fields, oneofs and reserved
declarations (parsed and ignored).
"""

from __future__ import annotations

import os
import re
import sys
from dataclasses import dataclass, field

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
PROTO_DIR = os.path.join(ROOT, "proto")

SCALARS = {
    "double", "float", "int32", "int64", "uint32", "uint64", "sint32", "sint64", "fixed32", "fixed64",
    "sfixed32", "sfixed64", "bool", "string", "bytes",
}


@dataclass
class Field:
    name: str
    number: int
    type: str  # scalar name or referenced type name (resolved later to a full name)
    label: str = ""  # "", "repeated", "optional"
    oneof: str | None = None
    map_key: str | None = None
    map_value: str | None = None
    full_type: str | None = None  # resolved full name for message/enum types
    is_enum: bool = False


@dataclass
class Enum:
    name: str
    full: str
    values: list[tuple[str, int]] = field(default_factory=list)


@dataclass
class Message:
    name: str
    full: str
    fields: list[Field] = field(default_factory=list)
    enums: list[Enum] = field(default_factory=list)
    oneofs: list[str] = field(default_factory=list)


@dataclass
class ProtoFile:
    path: str  # relative to PROTO_DIR
    package: str
    imports: list[str]
    enums: list[Enum]
    messages: list[Message]


_TOKEN = re.compile(r'\s+|//[^\n]*|/\*.*?\*/|"[^"]*"|[A-Za-z_][\w.]*|-?\d+|[{}=;<>,\[\]()]', re.S)


def _tokens(text: str) -> list[str]:
    out = []
    pos = 0
    while pos < len(text):
        m = _TOKEN.match(text, pos)
        if not m:
            raise SyntaxError(f"unexpected character {text[pos]!r} at {pos}")
        t = m.group(0)
        pos = m.end()
        if t.isspace() or t.startswith("//") or t.startswith("/*"):
            continue
        out.append(t)
    return out


class _Parser:
    def __init__(self, toks: list[str]):
        self.t = toks
        self.i = 0

    def peek(self) -> str | None:
        return self.t[self.i] if self.i < len(self.t) else None

    def take(self, want: str | None = None) -> str:
        tok = self.t[self.i]
        if want is not None and tok != want:
            raise SyntaxError(f"expected {want!r}, got {tok!r} (token {self.i})")
        self.i += 1
        return tok

    def skip_statement(self) -> None:
        while self.take() != ";":
            pass

    def parse_file(self, path: str) -> ProtoFile:
        pkg, imports, enums, msgs = "", [], [], []
        while self.peek() is not None:
            tok = self.take()
            if tok == "syntax":
                self.skip_statement()
            elif tok == "package":
                pkg = self.take()
                self.take(";")
            elif tok == "import":
                imports.append(self.take().strip('"'))
                self.take(";")
            elif tok == "option":
                self.skip_statement()
            elif tok == "enum":
                enums.append(self.parse_enum(pkg))
            elif tok == "message":
                msgs.append(self.parse_message(pkg))
            else:
                raise SyntaxError(f"unexpected {tok!r} at top level of {path}")
        return ProtoFile(path, pkg, imports, enums, msgs)

    def parse_enum(self, scope: str) -> Enum:
        name = self.take()
        e = Enum(name, f"{scope}.{name}")
        self.take("{")
        while self.peek() != "}":
            tok = self.take()
            if tok in ("reserved", "option"):
                self.skip_statement()
                continue
            self.take("=")
            e.values.append((tok, int(self.take())))
            if self.peek() == "[":
                while self.take() != "]":
                    pass
            self.take(";")
        self.take("}")
        return e

    def parse_message(self, scope: str) -> Message:
        name = self.take()
        m = Message(name, f"{scope}.{name}")
        self.take("{")
        self._body(m, None)
        self.take("}")
        return m

    def _body(self, m: Message, oneof: str | None) -> None:
        while self.peek() != "}":
            tok = self.take()
            if tok in ("reserved", "option"):
                self.skip_statement()
            elif tok == "enum":
                m.enums.append(self.parse_enum(m.full))
            elif tok == "message":
                raise SyntaxError("nested messages are not used by these schemas")
            elif tok == "oneof":
                oname = self.take()
                m.oneofs.append(oname)
                self.take("{")
                self._body(m, oname)
                self.take("}")
            elif tok == "map":
                self.take("<")
                k = self.take()
                self.take(",")
                v = self.take()
                self.take(">")
                fname = self.take()
                self.take("=")
                num = int(self.take())
                self.take(";")
                m.fields.append(Field(fname, num, "map", "repeated", oneof, map_key=k, map_value=v))
            else:
                label = ""
                if tok in ("repeated", "optional"):
                    label = tok
                    tok = self.take()
                ftype = tok
                fname = self.take()
                self.take("=")
                num = int(self.take())
                if self.peek() == "[":
                    while self.take() != "]":
                        pass
                self.take(";")
                m.fields.append(Field(fname, num, ftype, label, oneof))


def load_all(proto_dir: str = PROTO_DIR) -> dict[str, ProtoFile]:
    files = {}
    base = os.path.join(proto_dir, "everserve", "proto")
    for name in sorted(os.listdir(base)):
        if name.endswith(".proto"):
            rel = f"everserve/proto/{name}"
            with open(os.path.join(base, name)) as f:
                files[rel] = _Parser(_tokens(f.read())).parse_file(rel)
    _resolve(files)
    return files


def _resolve(files: dict[str, ProtoFile]) -> None:
    msgs, enums = {}, {}
    for pf in files.values():
        for e in pf.enums:
            enums[e.full] = e
        for m in pf.messages:
            msgs[m.full] = m
            for e in m.enums:
                enums[e.full] = e

    def lookup(name: str, scopes: list[str]) -> tuple[str, bool]:
        for sc in scopes:
            cand = f"{sc}.{name}" if sc else name
            if cand in msgs:
                return cand, False
            if cand in enums:
                return cand, True
        raise KeyError(f"unresolved type {name} in {scopes}")

    for pf in files.values():
        for m in pf.messages:
            scopes = [m.full, pf.package, ""]
            for f in m.fields:
                if f.type == "map":
                    if f.map_value not in SCALARS:
                        f.full_type, f.is_enum = lookup(f.map_value, scopes)
                elif f.type not in SCALARS:
                    f.full_type, f.is_enum = lookup(f.type, scopes)


# ---- Python descriptors ------------------------------------------------------------------------

def _camel(name: str) -> str:
    parts = name.split("_")
    return parts[0] + "".join(p[:1].upper() + p[1:] for p in parts[1:])


def build_python(files: dict[str, ProtoFile]):
    """Register every file in a private descriptor pool; returns {full_name: message class}."""
    from google.protobuf import descriptor_pb2, descriptor_pool, message_factory

    T = descriptor_pb2.FieldDescriptorProto
    stype = {
        "double": T.TYPE_DOUBLE, "float": T.TYPE_FLOAT, "int32": T.TYPE_INT32, "int64": T.TYPE_INT64,
        "uint32": T.TYPE_UINT32, "uint64": T.TYPE_UINT64, "sint32": T.TYPE_SINT32, "sint64": T.TYPE_SINT64,
        "fixed32": T.TYPE_FIXED32, "fixed64": T.TYPE_FIXED64, "sfixed32": T.TYPE_SFIXED32,
        "sfixed64": T.TYPE_SFIXED64, "bool": T.TYPE_BOOL, "string": T.TYPE_STRING, "bytes": T.TYPE_BYTES,
    }
    pool = descriptor_pool.DescriptorPool()

    def set_type(fd, type_name, full, is_enum):
        if type_name in stype:
            fd.type = stype[type_name]
        else:
            fd.type = T.TYPE_ENUM if is_enum else T.TYPE_MESSAGE
            fd.type_name = "." + full

    def add_enum(container, e: Enum):
        ed = container.add(name=e.name)
        for n, v in e.values:
            ed.value.add(name=n, number=v)

    order = []
    seen = set()

    def visit(path):
        if path in seen:
            return
        seen.add(path)
        for dep in files[path].imports:
            visit(dep)
        order.append(path)

    for p in files:
        visit(p)
    for path in order:
        pf = files[path]
        fdp = descriptor_pb2.FileDescriptorProto(name=path, package=pf.package, syntax="proto3")
        fdp.dependency.extend(pf.imports)
        for e in pf.enums:
            add_enum(fdp.enum_type, e)
        for m in pf.messages:
            md = fdp.message_type.add(name=m.name)
            for e in m.enums:
                add_enum(md.enum_type, e)
            oneof_index = {}
            for o in m.oneofs:
                oneof_index[o] = len(md.oneof_decl)
                md.oneof_decl.add(name=o)
            for f in m.fields:
                fd = md.field.add(name=f.name, number=f.number, json_name=_camel(f.name))
                if f.type == "map":
                    entry_name = "".join(p[:1].upper() + p[1:] for p in f.name.split("_")) + "Entry"
                    ent = md.nested_type.add(name=entry_name)
                    ent.options.map_entry = True
                    k = ent.field.add(name="key", number=1, json_name="key", label=T.LABEL_OPTIONAL)
                    set_type(k, f.map_key, None, False)
                    v = ent.field.add(name="value", number=2, json_name="value", label=T.LABEL_OPTIONAL)
                    set_type(v, f.map_value, f.full_type, f.is_enum)
                    fd.label = T.LABEL_REPEATED
                    fd.type = T.TYPE_MESSAGE
                    fd.type_name = f".{m.full}.{entry_name}"
                    continue
                fd.label = T.LABEL_REPEATED if f.label == "repeated" else T.LABEL_OPTIONAL
                set_type(fd, f.type, f.full_type, f.is_enum)
                if f.oneof is not None:
                    fd.oneof_index = oneof_index[f.oneof]
            # proto3 `optional`: a synthetic oneof per field, declared after the real ones
            for f, fd in zip(m.fields, md.field):
                if f.label == "optional":
                    fd.proto3_optional = True
                    fd.oneof_index = len(md.oneof_decl)
                    md.oneof_decl.add(name="_" + f.name)
        pool.Add(fdp)
    classes = {}
    for pf in files.values():
        for m in pf.messages:
            classes[m.full] = message_factory.GetMessageClass(pool.FindMessageTypeByName(m.full))
    return pool, classes


# ---- C++ ---------------------------------------------------------------------------------------

_CPP_SCALAR = {
    "double": "double", "float": "float", "int32": "int32_t", "int64": "int64_t", "uint32": "uint32_t",
    "uint64": "uint64_t", "sint32": "int32_t", "sint64": "int64_t", "fixed32": "uint32_t", "fixed64": "uint64_t",
    "sfixed32": "int32_t", "sfixed64": "int64_t", "bool": "bool", "string": "std::string", "bytes": "std::string",
}
_WIRE = {  # proto wire kinds
    "double": "F64", "float": "F32", "int32": "VARINT", "int64": "VARINT", "uint32": "VARINT", "uint64": "VARINT",
    "sint32": "ZIGZAG", "sint64": "ZIGZAG", "fixed32": "F32", "fixed64": "F64", "sfixed32": "F32", "sfixed64": "F64",
    "bool": "VARINT", "string": "LEN", "bytes": "LEN",
}


_CPP_KEYWORDS = {"class", "register", "default", "delete", "new", "operator", "private", "public", "template",
                 "this", "union", "virtual", "namespace", "auto", "case", "switch", "int", "long", "short", "char"}


def _cf(name: str) -> str:
    """C++ member name of a field (keywords get a trailing underscore)."""
    return name + "_" if name in _CPP_KEYWORDS else name


def _cpp_name(full: str) -> str:
    # everserve.signals.v1.Change -> signals::Change ; nested enums Foo.Bar -> Foo_Bar
    parts = full.split(".")
    pkg = parts[1]
    rest = [p for p in parts[3:]]
    return f"{pkg}::" + "_".join(rest)


def _field_cpp_type(f: Field) -> str:
    if f.type == "map":
        k = _CPP_SCALAR[f.map_key]
        v = _CPP_SCALAR.get(f.map_value) or (("int32_t" if f.is_enum else _cpp_name(f.full_type)))
        return f"std::map<{k}, {v}>"
    if f.type in _CPP_SCALAR:
        base = _CPP_SCALAR[f.type]
    elif f.is_enum:
        base = "int32_t"
    else:
        base = _cpp_name(f.full_type)
    if f.label == "repeated":
        return f"std::vector<{base}>"
    return base


def emit_cpp(files: dict[str, ProtoFile]) -> str:
    msgs = {m.full: m for pf in files.values() for m in pf.messages}
    enums = {e.full: e for pf in files.values() for e in pf.enums}
    for pf in files.values():
        for m in pf.messages:
            for e in m.enums:
                enums[e.full] = e
    # dependency order: a struct after every struct it holds by value
    order, state = [], {}

    def visit(name):
        if state.get(name) == 2:
            return
        if state.get(name) == 1:
            raise ValueError(f"recursive message {name}")
        state[name] = 1
        for f in msgs[name].fields:
            dep = f.full_type
            if dep in msgs and not f.is_enum:
                visit(dep)
        state[name] = 2
        order.append(name)

    for name in msgs:
        visit(name)
    out = []
    w = out.append
    w("// Generated by everserve_b200/proto/protogen.py from proto/everserve/proto/*.proto. Do not edit.")
    w("// Structs of the control-plane schemas with a proto3 binary codec (wire-compatible).")
    w("#pragma once")
    w("#include <cstdint>\n#include <map>\n#include <string>\n#include <vector>\n")
    w('#include "pbwire.h"\n')
    pkgs = sorted({full.split(".")[1] for full in list(msgs) + list(enums)})
    for pkg in pkgs:
        w(f"namespace {pkg} {{")
        for e in enums.values():
            if e.full.split(".")[1] != pkg:
                continue
            cname = _cpp_name(e.full).split("::")[1]
            w(f"enum {cname} : int32_t {{")
            for n, v in e.values:
                w(f"  {cname}_{n} = {v},")
            w("};")
        for name in order:
            if name.split(".")[1] == pkg:
                w(f"struct {_cpp_name(name).split('::')[1]};")
        w(f"}}  // namespace {pkg}")
    for name in order:
        m = msgs[name]
        pkg, cname = _cpp_name(name).split("::")
        w(f"namespace {pkg} {{")
        w(f"struct {cname} {{")
        for f in m.fields:
            ctype = _field_cpp_type(f)
            default = ""
            if f.label != "repeated" and f.type != "map" and (f.type in _CPP_SCALAR and f.type not in ("string", "bytes") or f.is_enum):
                default = "{}"
            w(f"  {ctype} {_cf(f.name)}{default};")
            if (f.label == "optional" or f.oneof is not None or (f.full_type in msgs and not f.is_enum)) and f.label != "repeated":
                w(f"  bool has_{f.name} = false;")
        w("  void encode(std::string& out) const;")
        w("  bool decode(const uint8_t* p, size_t n);")
        w("  std::string serialize() const { std::string s; encode(s); return s; }")
        w("  bool parse(const std::string& s) { return decode(reinterpret_cast<const uint8_t*>(s.data()), s.size()); }")
        w("};")
        w(f"}}  // namespace {pkg}")
    # codec bodies
    w("\nnamespace pbgen_detail {")
    w("using namespace pbwire;")
    w("}  // namespace pbgen_detail")
    for name in order:
        m = msgs[name]
        qual = _cpp_name(name)
        w(f"inline void {qual}::encode(std::string& out) const {{")
        w("  using namespace pbwire;")
        for f in m.fields:
            w("  " + _enc_field(f, msgs))
        w("}")
        w(f"inline bool {qual}::decode(const uint8_t* p, size_t n) {{")
        w("  using namespace pbwire;")
        w("  Reader r{p, p + n};")
        w("  while (r.p < r.end) {")
        w("    uint64_t tag_;")
        w("    if (!r.varint(tag_)) return false;")
        w("    const uint32_t num = (uint32_t)(tag_ >> 3), wt = (uint32_t)(tag_ & 7);")
        w("    switch (num) {")
        for f in m.fields:
            w(f"      case {f.number}: {{ {_dec_field(f, msgs)} break; }}")
        w("      default: if (!r.skip(wt)) return false;")
        w("    }")
        w("  }")
        w("  return true;")
        w("}")
    # decode then encode by full message name: the codec's check against other encoders
    w("\nnamespace pbgen {")
    w("// Decode `in` as the message `full` names (\"everserve.signals.v1.Change\") and encode it again;")
    w("// false for an unknown name or bytes the codec refuses.")
    w("inline bool roundtrip(const std::string& full, const std::string& in, std::string& out) {")
    for name in sorted(msgs):
        w(f'  if (full == "{name}") {{ {_cpp_name(name)} m; if (!m.parse(in)) return false; out = m.serialize(); return true; }}')
    w("  return false;")
    w("}")
    w("}  // namespace pbgen")
    return "\n".join(out) + "\n"


def _kind(t: str, is_enum: bool) -> str:
    if is_enum:
        return "VARINT"
    return _WIRE[t]


def _enc_field(f: Field, msgs) -> str:
    n = f.number
    fn = _cf(f.name)
    if f.type == "map":
        kt, vt = f.map_key, f.map_value
        vmsg = f.full_type in msgs and not f.is_enum
        venc = (f"{{ std::string sub; kv.second.encode(sub); put_len(e, 2, sub); }}" if vmsg else
                f"put_{_kind(vt, f.is_enum).lower()}(e, 2, kv.second);")
        return (f"for (const auto& kv : {fn}) {{ std::string e; put_{_kind(kt, False).lower()}(e, 1, kv.first); "
                f"{venc} put_len(out, {n}, e); }}")
    is_msg = f.full_type in msgs and not f.is_enum
    if f.label == "repeated":
        if is_msg:
            return f"for (const auto& v : {fn}) {{ std::string sub; v.encode(sub); put_len(out, {n}, sub); }}"
        k = _kind(f.type, f.is_enum)
        if k == "LEN":
            return f"for (const auto& v : {fn}) put_len(out, {n}, v);"
        return f"put_packed_{k.lower()}(out, {n}, {fn});"
    if is_msg:
        return f"if (has_{f.name}) {{ std::string sub; {fn}.encode(sub); put_len(out, {n}, sub); }}"
    k = _kind(f.type, f.is_enum).lower()
    explicit = f.label == "optional" or f.oneof is not None
    if explicit:
        return f"if (has_{f.name}) put_{k}(out, {n}, {fn});"
    if f.type in ("string", "bytes"):
        return f"if (!{fn}.empty()) put_len(out, {n}, {fn});"
    return f"if ({fn} != 0) put_{k}(out, {n}, {fn});"


def _dec_field(f: Field, msgs) -> str:
    is_msg = f.full_type in msgs and not f.is_enum
    fn = _cf(f.name)
    if f.type == "map":
        kt, vt = f.map_key, f.map_value
        vmsg = f.full_type in msgs and not f.is_enum
        ktype = _CPP_SCALAR[kt]
        vtype = _CPP_SCALAR.get(vt) or ("int32_t" if f.is_enum else _cpp_name(f.full_type))
        vdec = ("if (!get_msg(er, ewt, v)) return false;" if vmsg else
                f"if (!get_{_kind(vt, f.is_enum).lower()}(er, ewt, v)) return false;")
        return ("const uint8_t* b; size_t len; if (!r.bytes(b, len)) return false; Reader er{b, b + len}; "
                f"{ktype} k{{}}; {vtype} v{{}}; while (er.p < er.end) {{ uint64_t ek; if (!er.varint(ek)) return false; "
                "const uint32_t ewt = (uint32_t)(ek & 7); "
                f"if ((ek >> 3) == 1) {{ if (!get_{_kind(kt, False).lower()}(er, ewt, k)) return false; }} "
                f"else if ((ek >> 3) == 2) {{ {vdec} }} else if (!er.skip(ewt)) return false; }} "
                f"{fn}[k] = v;")
    if f.label == "repeated":
        if is_msg:
            return f"{fn}.emplace_back(); if (!get_msg(r, wt, {fn}.back())) return false;"
        k = _kind(f.type, f.is_enum)
        if k == "LEN":
            return f"{fn}.emplace_back(); if (!get_len(r, wt, {fn}.back())) return false;"
        return f"if (!get_repeated_{k.lower()}(r, wt, {fn})) return false;"
    if is_msg:
        return f"if (!get_msg(r, wt, {fn})) return false; has_{f.name} = true;"
    k = _kind(f.type, f.is_enum).lower()
    tail = f" has_{f.name} = true;" if (f.label == "optional" or f.oneof is not None) else ""
    return f"if (!get_{k}(r, wt, {fn})) return false;{tail}"


def main(argv: list[str]) -> None:
    files = load_all()
    if len(argv) >= 2 and argv[0] == "--cpp":
        text = emit_cpp(files)
        os.makedirs(os.path.dirname(os.path.abspath(argv[1])), exist_ok=True)
        old = open(argv[1]).read() if os.path.exists(argv[1]) else None
        if old != text:
            with open(argv[1], "w") as f:
                f.write(text)
        return
    for path, pf in files.items():
        print(path, pf.package, len(pf.messages), "messages", len(pf.enums), "enums")


if __name__ == "__main__":
    main(sys.argv[1:])
