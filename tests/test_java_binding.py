"""The Java FFM binding module (jax4j_b200/java/jax4j-engine-b200) against the C ABI it binds.

No JDK is installed on the build machine, so the Java sources are checked here structurally:
every downcall names a function that include/jax4j_b200.h declares and libjax4j_b200.so exports,
with an argument layout list whose length and kinds (int, int64/size_t/j4b_buf, float, double,
pointer) match the C parameter list; the service files name classes that exist; the Op and
AadOp ordinals the binding passes are the engine's op codes."""
import ctypes
import pathlib
import re

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
MODULE = ROOT / "jax4j_b200" / "java" / "jax4j-engine-b200"
SOURCES = sorted((MODULE / "src" / "main" / "java").rglob("*.java"))
LETTER = {"JAVA_INT": "I", "JAVA_LONG": "L", "JAVA_FLOAT": "F", "JAVA_DOUBLE": "D", "ADDRESS": "P",
          "I": "I", "L": "L", "F": "F", "D": "D", "P": "P"}


def c_signatures() -> dict:
    text = (ROOT / "include" / "jax4j_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    out = {}
    for name, params in re.findall(r"\bint\s+(j4b_\w+)\s*\(([^)]*)\)\s*;", text):
        kinds = []
        for p in (x.strip() for x in params.split(",")):
            if not p or p == "void":
                continue
            if "*" in p or p.split()[0] in ("j4b_stream", "j4b_qweight_t", "j4b_aad_t", "j4b_qplan_t"):
                kinds.append("P")
            elif p.split()[0] in ("j4b_buf", "int64_t", "uint64_t", "size_t"):
                kinds.append("L")
            elif p.split()[0] == "int":
                kinds.append("I")
            elif p.split()[0] == "float":
                kinds.append("F")
            elif p.split()[0] == "double":
                kinds.append("D")
            else:
                raise AssertionError(f"unmapped C parameter type in {name}: {p}")
        out[name] = "".join(kinds)
    return out


def java_downcalls() -> list:
    """(file, function, layout letters) for every call(...) and fn(...) in the module."""
    found = []
    for src in SOURCES:
        text = src.read_text()
        arrays = {n: "".join(LETTER[x.strip()] for x in body.split(",") if x.strip())
                  for n, body in re.findall(r"MemoryLayout\[\]\s+(\w+)\s*=\s*sig\(([^)]*)\)", text)}
        for name, arg in re.findall(r'\bcall\(\s*(?:entry|"(j4b_\w+)")\s*,\s*(sig\([^)]*\)|\w+)', text):
            if not name:
                continue
            if arg.startswith("sig("):
                letters = "".join(LETTER[x.strip()] for x in arg[4:-1].split(",") if x.strip())
            else:
                letters = arrays[arg]
            found.append((src.name, name, letters))
        for name, rest in re.findall(r'\bfn\(\s*"(j4b_\w+)"((?:\s*,\s*\w+)*)\s*\)', text):
            found.append((src.name, name, "".join(LETTER[x.strip()] for x in rest.split(",") if x.strip())))
        # call(entry, ...) forwards a name chosen at the call site: resolve those names too
        for helper, layout in (("axisReduce", "AXIS"), ("conv", "CONV")):
            for name in re.findall(helper + r'\(\s*"(j4b_\w+)"', text):
                found.append((src.name, name, arrays[layout]))
    return found


def test_every_downcall_matches_the_c_declaration():
    sigs = c_signatures()
    calls = java_downcalls()
    assert len({c[1] for c in calls}) >= 40
    for src, name, letters in calls:
        assert name in sigs, f"{src}: {name} is not declared in include/jax4j_b200.h"
        assert letters == sigs[name], f"{src}: {name} binds ({letters}), the header declares ({sigs[name]})"


def test_every_bound_function_is_exported(oracle):
    from jax4j_b200 import _lib
    lib = ctypes.CDLL(_lib.LIB_PATH)
    for _, name, _ in java_downcalls():
        assert hasattr(lib, name), f"{name} is not exported by {_lib.LIB_PATH}"


def test_service_files_name_existing_provider_classes():
    services = MODULE / "src" / "main" / "resources" / "META-INF" / "services"
    wanted = {"com.nablatensor.jax4j.tensor.spi.ComputeBackend": "implements ComputeBackend, QuantizedOps",
              "com.nablatensor.jax4j.engine.AadEngine": "extends B200AadEngines.Base"}
    for service, marker in wanted.items():
        names = [n.strip() for n in (services / service).read_text().splitlines() if n.strip()]
        assert names
        for cls in names:
            path = MODULE / "src" / "main" / "java" / (cls.replace(".", "/") + ".java")
            text = path.read_text()
            simple = cls.rsplit(".", 1)[1]
            assert f"public final class {simple}" in text and marker in text
            assert re.search(rf"public {simple}\(\)", text) or "public B200Backend" not in text


def test_op_codes_are_the_reference_ordinals():
    """Op (tensor/Op.java) and AadOp ordinals are what the binding passes as op codes."""
    from jax4j_b200 import aad, expr
    ops = ["ADD", "SUB", "MUL", "DIV", "MAX", "MIN", "NEG", "EXP", "LOG", "SQRT", "RSQRT", "TANH",
           "SIGMOID", "RELU", "ABS", "SIGN"]
    assert [expr.OP[o] for o in ops] == list(range(16))
    assert [m.name for m in aad.AadOp] == ["CONST", "INPUT", "RANDN", "RANDU", "ADD", "SUB", "MUL", "DIV",
                                          "NEG", "EXP", "LOG", "SQRT", "MAX", "MIN", "ABS"]


@pytest.mark.parametrize("path", SOURCES, ids=lambda p: p.name)
def test_sources_are_balanced_and_packaged(path):
    text = path.read_text()
    stripped = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    stripped = re.sub(r'"(?:\\.|[^"\\])*"', '""', re.sub(r"//[^\n]*", "", stripped))
    for a, b in ("()", "{}", "[]"):
        assert stripped.count(a) == stripped.count(b), f"{path.name}: unbalanced {a}{b}"
    assert text.startswith("package com.nablatensor.jax4j.backend.b200;")


def test_one_call_fused_tape_layout_plans(oracle):
    """B200Backend.fused serialises an expression as a one-call tape: header, n input shapes and
    the output shape (input 0's), inputs 0..n-1, output n, then the call (opcode 2, out n, n ins,
    postfix program with scalars as signed lo32/hi32). The engine's planner accepts that layout
    (j4b_tape_dryrun: NVRTC, no device) for x * y + 3 over two [4, 5] inputs."""
    import numpy as np
    import struct
    from jax4j_b200 import _lib
    from jax4j_b200.jit import TAPE_MAGIC
    lo, hi = struct.unpack("<ii", struct.pack("<d", 3.0))
    program = [0, 0, 0, 1, 2, _lib.OP["MUL"], 3, _lib.OP["ADD"], lo, hi]
    n, dims = 2, [4, 5]
    words = [TAPE_MAGIC, n + 1, n, 1, 1]
    for _ in range(n + 1):
        words += [len(dims)] + dims
    words += list(range(n)) + [n]
    words += [2, n, n] + list(range(n)) + [len(program)] + program
    w = np.asarray(words, np.int64)
    st = _lib.TapeStats()
    size = ctypes.c_size_t()
    _lib.call("j4b_tape_dryrun", w.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)), w.size, ctypes.byref(st),
              None, 0, ctypes.byref(size))
    assert (st.calls, st.groups) == (1, 1)


def test_backend_overrides_every_spi_method_with_its_signature():
    """B200Backend declares every ComputeBackend and QuantizedOps method with the reference's
    parameter and return types (tests/golden/spi_signatures.json, generated from the SPI sources
    by tests/golden/make_spi_signatures.py). Only `program` and `custom` keep the SPI defaults:
    those evaluate through the backend's own calls, which are all device-local here."""
    import json
    spi = json.loads((ROOT / "tests" / "golden" / "spi_signatures.json").read_text())
    src = (MODULE / "src" / "main" / "java" / "com" / "nablatensor" / "jax4j" / "backend" / "b200" /
           "B200Backend.java").read_text()
    declared = {}
    for ret, name, params in re.findall(r"public\s+([\w.<>\[\], ]+?)\s+(\w+)\(([^)]*)\)", src):
        types = [" ".join(p.split()).rsplit(" ", 1)[0] for p in params.split(",") if p.strip()]
        declared.setdefault(name, []).append((ret.strip(), types))
    assert len(spi["ComputeBackend"]) == 37 and len(spi["QuantizedOps"]) == 5
    for iface in ("ComputeBackend", "QuantizedOps"):
        for m in spi[iface]:
            if m["name"] in ("program", "custom"):
                continue
            assert m["name"] in declared, f"{iface}.{m['name']} is not implemented"
            assert (m["returns"], m["params"]) in declared[m["name"]], \
                f"{iface}.{m['name']}: {declared[m['name']]} vs ({m['returns']}, {m['params']})"


def test_aad_providers_implement_the_engine_interfaces():
    """The AadEngine methods are declared by the providers' shared base, and B200AadExecutable
    declares the AadExecutable methods AbstractAadExecutable leaves open (engineName, replay)
    plus its close and compileSeconds, all with the reference's types."""
    import json
    spi = json.loads((ROOT / "tests" / "golden" / "spi_signatures.json").read_text())
    pkg = MODULE / "src" / "main" / "java" / "com" / "nablatensor" / "jax4j" / "backend" / "b200"

    def declared(path):
        out = {}
        for ret, name, params in re.findall(r"public\s+(?:synchronized\s+)?([\w.<>\[\], ]+?)\s+(\w+)\(([^)]*)\)",
                                            path.read_text()):
            types = [" ".join(p.split()).rsplit(" ", 1)[0] for p in params.split(",") if p.strip()]
            out.setdefault(name, []).append((ret.strip(), types))
        return out

    engines, exe = declared(pkg / "B200AadEngines.java"), declared(pkg / "B200AadExecutable.java")
    for m in spi["AadEngine"]:
        assert (m["returns"], m["params"]) in engines.get(m["name"], []), f"AadEngine.{m['name']}"
    want = {m["name"]: m for m in spi["AadExecutable"]}
    for name in ("engineName", "replay", "close", "compileSeconds"):
        assert (want[name]["returns"], want[name]["params"]) in exe.get(name, []), f"AadExecutable.{name}"


# JDK and JUnit members the module calls (java.lang.foreign, java.lang.invoke, java.util,
# java.util.stream, java.lang.ref, Math/Long/Double/Integer/System, enum values/ordinal/name,
# JUnit's DynamicTest)
JDK_NAMES = {
    "of", "add", "get", "ofConfined", "allocate", "allocateFrom", "size", "equals", "toArray", "stream",
    "toString", "flatMap", "map", "byteSize", "append", "addAll", "values", "register", "nanoTime",
    "multiplyExact", "libraryLookup", "global", "getString", "dynamicTest", "create", "contains",
    "computeIfAbsent", "compareAndSet", "clean", "asLongStream", "trim", "sqrt", "sin", "cos", "exp",
    "remove", "parseLong", "orElseThrow", "ofArray", "noneOf", "newKeySet", "nativeLinker", "mapToLong",
    "isNative", "isEmpty", "invokeWithArguments", "invokeExact", "getProperty", "getInteger", "getAtIndex",
    "find", "downcallHandle", "doubleToRawLongBits", "copyOfRange", "copy", "clone", "asSlice", "arraycopy",
    "max", "ordinal", "name", "longValue", "valueOf",
}


def test_every_called_member_exists_in_the_reference_or_the_jdk():
    """Each `.name(` call in the module names a member of an imported reference class (from the
    reference sources, tests/golden/spi_signatures.json), of the module itself, or of the JDK /
    JUnit APIs listed above: a mistyped reference accessor fails here rather than at a
    maintainer's first compile."""
    import json
    ref = json.loads((ROOT / "tests" / "golden" / "spi_signatures.json").read_text())["reference_names"]
    known = set().union(*ref.values()) | JDK_NAMES
    sources = sorted((MODULE / "src").rglob("*.java"))
    own = set()
    for src in sources:
        own |= set(re.findall(r"\b(\w+)\s*\([^;{]*\)\s*(?:throws [\w, ]+)?\{", src.read_text()))
    for src in sources:
        text = re.sub(r'"(?:\\.|[^"\\])*"', '""', re.sub(r"//[^\n]*|/\*.*?\*/", "", src.read_text(), flags=re.S))
        for name in set(re.findall(r"\.(\w+)\(", text)):
            assert name in known or name in own, f"{src.name}: .{name}( is not a known member"
