"""The Java drop-in (java/nablatensor-engine-b200) against the C ABI and the
reference's engine SPI, without a JDK.

No JDK exists on this host or on the GPU box, so the module cannot be
compiled here.  What can go wrong between it and its two neighbours is
checked from the sources instead:
  - every FFM downcall descriptor in B200Native.java matches the prototype
    in include/nabla_b200.h (arity, and int32 / int64 / double / pointer per
    argument and result), and every struct layout names the header's fields
    in order at the C offsets;
  - every method marked @Override exists, with the same parameter types, in
    the reference interface or base class it overrides and is not final or
    private there; the methods and fields the module calls on the reference's
    types exist (tests/golden/java_spi.json, generated from the reference
    sources by tests/golden/make_java_spi.py);
  - the op codes the module passes (AadOpEnum ordinals) are the header's
    enum order; the engine options it accepts are the Python mirror's; its
    priority is the Python mirror's; its service file names the engine class.
"""
import json
import os
import re

import pytest

from nablatensor_b200 import _lib
from nablatensor_b200.engine import _ENGINE_FLAGS, _ENGINE_KEYS, CudaAadEngine

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
MODULE = os.path.join(ROOT, "java", "nablatensor-engine-b200")
PKG = os.path.join(MODULE, "src", "main", "java", "com", "nablatensor", "engine", "b200")
HEADER = os.path.join(ROOT, "include", "nabla_b200.h")


def _java(name):
    with open(os.path.join(PKG, name)) as f:
        text = f.read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return re.sub(r"//[^\n]*", "", text)


@pytest.fixture(scope="module")
def spi():
    with open(os.path.join(ROOT, "tests", "golden", "java_spi.json")) as f:
        return json.load(f)


def _c_prototypes():
    with open(HEADER) as f:
        text = re.sub(r"/\*.*?\*/", "", f.read(), flags=re.S)
    protos = {}
    for ret, name, params in re.findall(r"^(int|void|const char\*)\s+(nt_\w+)\((.*?)\);", text, re.S | re.M):
        kinds = [] if params.strip() in ("", "void") else [_c_kind(p) for p in params.split(",")]
        protos[name] = (_c_kind(ret + " r"), kinds)
    return protos


def _c_kind(decl):
    decl = " ".join(decl.split())
    if "*" in decl or "[" in decl:
        return "ADDRESS"
    base = decl.rsplit(" ", 1)[0]
    if base in ("int32_t", "uint32_t", "int"):
        return "JAVA_INT"
    if base in ("uint64_t", "int64_t", "size_t"):
        return "JAVA_LONG"
    if base == "double":
        return "JAVA_DOUBLE"
    if base == "void":
        return "void"
    raise AssertionError(f"unmapped C type in {decl!r}")


def _downcalls():
    text = _java("B200Native.java")
    calls = {}
    for name, kind, args in re.findall(r'fn\("(nt_\w+)",\s*FunctionDescriptor\.(of|ofVoid)\(([^;]*?)\)\);', text,
                                       re.S):
        layouts = [a.strip() for a in args.split(",") if a.strip()]
        ret = "void" if kind == "ofVoid" else layouts.pop(0)
        calls[name] = (ret, layouts)
    return calls


def test_every_downcall_matches_its_c_prototype():
    protos, calls = _c_prototypes(), _downcalls()
    assert len(calls) >= 14
    for name, (ret, args) in calls.items():
        assert name in protos, f"{name} is not declared in nabla_b200.h"
        want_ret, want_args = protos[name]
        assert ret == want_ret, (name, ret, want_ret)
        assert args == want_args, (name, args, want_args)


def _header_fields(struct):
    with open(HEADER) as f:
        text = f.read()
    body = re.search(r"typedef struct " + struct + r" \{(.*?)\} " + struct + ";", text, re.S).group(1)
    body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
    return [re.search(r"(\w+)\s*;", line).group(1) for line in body.split("\n") if ";" in line]


@pytest.mark.parametrize("layout,struct,cls", [("TAPE", "nt_tape", _lib.NtTape),
                                               ("OPTIONS", "nt_options", _lib.NtOptions)])
def test_struct_layouts_name_the_header_fields_at_the_c_offsets(layout, struct, cls):
    text = _java("B200Native.java")
    body = re.search(r"StructLayout " + layout + r" = MemoryLayout\.structLayout\((.*?)\);", text, re.S).group(1)
    items = re.findall(r'(JAVA_INT|ADDRESS|JAVA_LONG|JAVA_DOUBLE)\.withName\("(\w+)"\)|paddingLayout\((\d+)\)', body)
    sizes = {"JAVA_INT": 4, "ADDRESS": 8, "JAVA_LONG": 8, "JAVA_DOUBLE": 8}
    offsets, at = {}, 0
    for kind, name, pad in items:
        if pad:
            at += int(pad)
            continue
        assert at % sizes[kind] == 0, f"{name} misaligned in the Java layout"
        offsets[name] = at
        at += sizes[kind]
    assert list(offsets) == _header_fields(struct)
    for name, _ in cls._fields_:
        assert offsets[name] == getattr(cls, name).offset, (layout, name)
    assert at == _lib.ctypes.sizeof(cls)


def _overrides(name):
    """(method, parameter types) of every @Override in a source file."""
    text = _java(name)
    out = []
    for m in re.finditer(r"@Override\s+(?:public|protected)\s+[\w<>\[\].]+\s+(\w+)\(([^)]*)\)", text):
        params = [re.sub(r"\s+\w+$", "", p.strip()).replace(" ", "") for p in m.group(2).split(",") if p.strip()]
        out.append((m.group(1), params))
    return out


@pytest.mark.parametrize("source,bases", [
    ("B200AadEngine.java", ["AadEngine"]),
    ("B200AadExecutable.java", ["AbstractAadExecutable", "AadExecutable"]),
])
def test_overrides_exist_in_the_reference_spi_and_are_overridable(spi, source, bases):
    found = _overrides(source)
    assert found
    for method, params in found:
        decls = [m for b in bases for m in spi["classes"][b]["methods"] if m["name"] == method]
        assert decls, f"{source}: {method} overrides nothing in {bases}"
        match = [m for m in decls if m["params"] == params]
        assert match, f"{source}: {method}{params} has no matching signature in {bases}: {decls}"
        for m in match:
            assert "final" not in m["modifiers"] and "private" not in m["modifiers"] \
                and "static" not in m["modifiers"], (method, m)


def test_the_executable_overrides_the_chunk_budget_and_leaves_replay_safe_to_the_base(spi):
    names = [m for m, _ in _overrides("B200AadExecutable.java")]
    assert "defaultMaxChunkSeconds" in names and "replay" in names
    base = {m["name"]: m for m in spi["classes"]["AbstractAadExecutable"]["methods"]}
    assert "final" in base["replaySafe"]["modifiers"] and "replaySafe" not in names
    assert "protected" in base["defaultMaxChunkSeconds"]["modifiers"]


def test_calls_into_the_reference_types_exist(spi):
    text = _java("B200AadExecutable.java") + _java("B200AadEngine.java")
    cls = spi["classes"]
    methods = lambda c: {m["name"] for m in cls[c]["methods"]}  # noqa: E731
    fields = lambda c: {f["name"] for f in cls[c]["fields"]}  # noqa: E731
    for m in set(re.findall(r"\btape\.(\w+)\(", text)):
        assert m in methods("AadTape"), f"AadTape.{m}"
    for m in set(re.findall(r"\boptions\.(\w+)\(", text)):
        assert m in methods("AadOptions"), f"AadOptions.{m}"
    for f_ in set(re.findall(r"\bf\.(\w+)\b(?!\()", text)) - {"size"}:
        assert f_ in fields("FlatTape"), f"FlatTape.{f_}"
    assert "size" in methods("FlatTape")
    for f_ in set(re.findall(r"\bt\.(value|sumsq|gradient)\b", text)):
        assert f_ in fields("AadTotals")
    assert "toResult" in methods("AadTotals")
    assert "maxLaunchSeconds" in methods("GpuAadExecutable")
    base_fields = {f["name"]: f for f in cls["AbstractAadExecutable"]["fields"]}
    for used in ("tape", "inputs"):
        assert used in base_fields and "private" not in base_fields[used]["modifiers"]
    assert "checkOpen" in methods("AbstractAadExecutable")
    for absent in ("isClosed(", "rethrow("):  # not part of the reference base class
        assert absent not in text


def test_op_codes_are_the_header_enum_order(spi):
    with open(HEADER) as f:
        text = f.read()
    body = re.search(r"enum nt_op \{(.*?)\};", text, re.S).group(1)
    header = [name[3:] for name, _ in re.findall(r"(NT_\w+)\s*=\s*(\d+)", body)]
    assert header == spi["AadOpEnum"]
    assert ".ordinal()" in _java("B200AadExecutable.java")


def test_engine_options_priority_and_service_file():
    text = _java("B200AadExecutable.java")
    keys = set(re.findall(r'case "(\w+)" ->', text))
    assert keys == set(_ENGINE_KEYS) | set(_ENGINE_FLAGS) - {"accRegisters"} | {"device"}
    prio = int(re.search(r"PRIORITY = (\d+);", _java("B200AadEngine.java")).group(1))
    assert prio == CudaAadEngine().priority() > 100  # found before the reference's cuda engine (100)
    with open(os.path.join(MODULE, "src", "main", "resources", "META-INF", "services",
                           "com.nablatensor.engine.AadEngine")) as f:
        assert f.read().strip() == "com.nablatensor.engine.b200.B200AadEngine"
    assert "public final class B200AadEngine implements AadEngine" in _java("B200AadEngine.java")
