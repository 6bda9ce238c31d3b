"""Regenerates tests/golden/spi_signatures.json from the reference checkout (run in the build
container, where the reference tree is mounted): the method declarations of the engine SPI the
Java binding module implements.

  ComputeBackend  <- jax4j-core/src/main/java/com/nablatensor/jax4j/tensor/spi/ComputeBackend.java
  QuantizedOps    <- jax4j-core/src/main/java/com/nablatensor/jax4j/tensor/spi/QuantizedOps.java
  AadEngine       <- jax4j-core/src/main/java/com/nablatensor/jax4j/engine/AadEngine.java
  AadExecutable   <- jax4j-core/src/main/java/com/nablatensor/jax4j/engine/AadExecutable.java

Each entry is {name, returns, params (simple type names), default (has a default body)};
private and static helpers are skipped.

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


def main(ref_root: str) -> None:
    fixture = {iface: parse(os.path.join(ref_root, d, iface + ".java")) for iface, d in SOURCES.items()}
    with open(os.path.join(HERE, "spi_signatures.json"), "w") as f:
        json.dump(fixture, f, indent=1)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("JAX4J_REF", "."))
