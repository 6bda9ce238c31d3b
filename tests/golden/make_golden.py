"""Regenerates the committed golden fixtures from the reference checkout (run in the build
container, where the reference tree is mounted; the GPU box only reads the JSON).

  jax_parity.json  <- jax4j-core/src/test/resources/jax-parity.properties (JAX 0.11.2 CPU values,
                      produced by the reference's python/jax_parity.py)
  kats.json        <- known-answer tests read from the reference's test sources
                      (CudaTensorTest.java:19-58, VmapTest.java:10-19, JitTest.java:16-43,
                      TransformsTest.java:14-32): inputs and expected values, transcribed below
                      with the file:line they come from.

Usage: python tests/golden/make_golden.py /path/to/jax4j
"""
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def parse_properties(path):
    out = {}
    with open(path) as f:
        for line in f:
            line = line.strip()
            if not line or line.startswith("#") or "=" not in line:
                continue
            k, v = line.split("=", 1)
            out[k] = v
    return out


def main(ref_root):
    props = parse_properties(os.path.join(
        ref_root, "jax4j-core/src/test/resources/jax-parity.properties"))
    fixture = {"source": "jax4j-core/src/test/resources/jax-parity.properties",
               "jax.version": props["jax.version"]}
    for k, v in props.items():
        if k in ("jax.version", "platform"):
            continue
        fixture[k] = [float(x) for x in v.split(",")]
    with open(os.path.join(HERE, "jax_parity.json"), "w") as f:
        json.dump(fixture, f, indent=1)
    # Known answers (values as they appear in the cited reference tests).
    kats = {
        "elementwise_and_sum": {"src": "CudaTensorTest.java:19-25", "x": [1, 2, 3, 4],
                                "y=x*x+3": [4, 7, 12, 19], "sum": 42},
        "matmul": {"src": "CudaTensorTest.java:27-33", "a": [[1, 2, 3], [4, 5, 6]],
                   "b": [[7, 8], [9, 10], [11, 12]], "c": [[58, 64], [139, 154]]},
        "fill": {"src": "CudaTensorTest.java:35-40", "value": -2.5, "n": 3},
        "compiled_replay": {"src": "CudaTensorTest.java:42-52", "x1": [1, 2], "y1": [4, 7],
                            "x2": [3, 4], "y2": [12, 19]},
        "compiled_grad_sum_sq": {"src": "CudaTensorTest.java:54-58", "x": [1, 2, 3],
                                 "grad": [2, 4, 6]},
        "vmap_sum_sq": {"src": "VmapTest.java:10-19", "x": [[1, 2, 3], [4, 5, 6]],
                        "out": [14, 77], "grad": [2, 4, 6, 8, 10, 12]},
        "jit_tanh": {"src": "JitTest.java:16-25", "x": [3, 4], "y=tanh(x*x+3)": "tanh([12,19])"},
        "jit_axis_boundary": {"src": "JitTest.java:26-31", "x": [1, 2], "bias": [10, 20],
                              "y": [12, 25]},
    }
    with open(os.path.join(HERE, "kats.json"), "w") as f:
        json.dump(kats, f, indent=1)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("JAX4J_REF", "."))
