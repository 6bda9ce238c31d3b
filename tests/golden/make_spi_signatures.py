"""Regenerates tests/golden/spi_signatures.json from the reference checkout (run in the build
container, where the reference tree is mounted): the method declarations of the engine SPI the
Java binding module implements.

  ComputeBackend  <- jax4j-core/src/main/java/com/nablatensor/jax4j/tensor/spi/ComputeBackend.java
  QuantizedOps    <- jax4j-core/src/main/java/com/nablatensor/jax4j/tensor/spi/QuantizedOps.java
  AadEngine       <- jax4j-core/src/main/java/com/nablatensor/jax4j/engine/AadEngine.java
  AadExecutable   <- jax4j-core/src/main/java/com/nablatensor/jax4j/engine/AadExecutable.java

Each entry is {name, returns, params (simple type names), default (has a default body)};
private and static helpers are skipped.

  reference_names <- the non-private member names (methods, record components) of every
                     reference class the module imports, for the check that each reference
                     method the module calls exists.

Usage: python tests/golden/make_spi_signatures.py /path/to/jax4j
"""
import json
import os
import re
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SOURCES = {"ComputeBackend": "jax4j-core/src/main/java/com/nablatensor/jax4j/tensor/spi",
           "QuantizedOps": "jax4j-core/src/main/java/com/nablatensor/jax4j/tensor/spi",
           "AadEngine": "jax4j-core/src/main/java/com/nablatensor/jax4j/engine",
           "AadExecutable": "jax4j-core/src/main/java/com/nablatensor/jax4j/engine"}
DECL = re.compile(r"^\s*(default\s+)?([A-Za-z_][\w.<>\[\], ]*?)\s+(\w+)\(([^)]*)\)\s*(;|\{)", re.M)


def simple(t: str) -> str:
    t = " ".join(t.split())
    return t.rsplit(".", 1)[-1] if "." in t and "<" not in t else t


def parse(path: str) -> list:
    text = open(path).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    text = re.sub(r"//[^\n]*", "", text)
    out = []
    for m in DECL.finditer(text):
        ret, name = m.group(2).strip(), m.group(3)
        if ret.startswith(("private", "static", "return", "new", "throw", "else")) or name in ("if", "for", "while", "switch"):
            continue
        params = [simple(p.rsplit(" ", 1)[0]) for p in (x.strip() for x in m.group(4).split(",")) if p]
        out.append({"name": name, "returns": simple(ret), "params": params, "default": bool(m.group(1))})
    return out


CORE = "jax4j-core/src/main/java/"
IMPORTED = ["com.nablatensor.jax4j.engine.AadEngine", "com.nablatensor.jax4j.engine.AadExecutable",
            "com.nablatensor.jax4j.engine.AadOptions", "com.nablatensor.jax4j.engine.AadRecorder",
            "com.nablatensor.jax4j.engine.AadResult", "com.nablatensor.jax4j.engine.AadTape",
            "com.nablatensor.jax4j.engine.AbstractAadExecutable", "com.nablatensor.jax4j.engine.SDouble",
            "com.nablatensor.jax4j.engine.cpu.CpuAadEngine", "com.nablatensor.jax4j.tensor.BackendRegistry",
            "com.nablatensor.jax4j.tensor.ConvSpec", "com.nablatensor.jax4j.tensor.DType",
            "com.nablatensor.jax4j.tensor.Device", "com.nablatensor.jax4j.tensor.DeviceType",
            "com.nablatensor.jax4j.tensor.Jit", "com.nablatensor.jax4j.tensor.Op",
            "com.nablatensor.jax4j.tensor.QuantType", "com.nablatensor.jax4j.tensor.Shape",
            "com.nablatensor.jax4j.tensor.Tensor", "com.nablatensor.jax4j.tensor.Tensors",
            "com.nablatensor.jax4j.tensor.Transforms", "com.nablatensor.jax4j.tensor.expr.Expr",
            "com.nablatensor.jax4j.tensor.spi.ComputeBackend", "com.nablatensor.jax4j.tensor.spi.DeviceBuffer",
            "com.nablatensor.jax4j.tensor.spi.QuantizedOps"]
MEMBER = re.compile(r"^\s*(?:(?:public|protected|static|final|default|abstract|synchronized)\s+)*"
                    r"(?:<[^>]*>\s*)?[A-Za-z_][\w.<>\[\], ?]*\s+(\w+)\s*\(", re.M)
RECORD = re.compile(r"\brecord\s+\w+\s*\(([^)]*)\)")


def member_names(path: str) -> list:
    text = open(path).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    text = re.sub(r"//[^\n]*", "", text)
    names = set()
    for line_m in MEMBER.finditer(text):
        line = text[line_m.start():line_m.end()]
        if "private" not in line.split("(")[0] and line_m.group(1) not in ("if", "for", "while", "switch", "return", "new"):
            names.add(line_m.group(1))
    for comps in RECORD.findall(text):
        for c in comps.split(","):
            if c.strip():
                names.add(c.split()[-1])
    return sorted(names)


def main(ref_root: str) -> None:
    fixture = {iface: parse(os.path.join(ref_root, d, iface + ".java")) for iface, d in SOURCES.items()}
    fixture["reference_names"] = {cls: member_names(os.path.join(ref_root, CORE, cls.replace(".", "/") + ".java"))
                                  for cls in IMPORTED}
    with open(os.path.join(HERE, "spi_signatures.json"), "w") as f:
        json.dump(fixture, f, indent=1)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("JAX4J_REF", "."))
