"""Regenerates the GGUF block-format fixtures from llama.cpp's own Python package `gguf`
(version 0.19.0, the one installed in the build image: gguf/quants.py holds ggml's published
block codecs, gguf/gguf_writer.py the file writer). The reference (jax4j) has no implementation
of Q8_0, Q4_K or Q6_K, only their geometry (core/tensor/QuantType.java:8-10), and no vendored
ggml; these fixtures pin the engine's and the oracle's codecs to ggml's own. The GPU box only
reads the committed outputs.

Writes, next to this script:
  gguf_vectors.npz   per type T in (Q8_0, Q4_0, Q4_K, Q6_K):
                       T_raw, T_raw_deq      random blocks (random codes, random f16 scales
                                             including negative and subnormal ones) and gguf's
                                             dequantisation of them, [rows, cols] float32
                     per type T in (Q8_0, Q4_0) (gguf 0.19 has encoders only for these):
                       T_w, T_blocks, T_deq  seeded weights with edge-case rows (zeros, a single
                                             spike, constant, rounding ties, large magnitude),
                                             gguf's encoding of them and its dequantisation
  gguf_writer.gguf   a file written by gguf.GGUFWriter: the raw Q8_0/Q4_0/Q4_K/Q6_K blocks
                     above as rank-2 tensors plus F32/F16 tensors and metadata of each kind

Usage: python tests/golden/make_gguf_vectors.py
"""
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

# ggml type id, block elements, block bytes, offsets of the f16 scale fields inside a block
TYPES = {"Q8_0": (8, 32, 34, (0,)), "Q4_0": (2, 32, 18, (0,)),
         "Q4_K": (12, 256, 144, (0, 2)), "Q6_K": (14, 256, 210, (208,))}
RAW_SHAPE = {"Q8_0": (12, 128), "Q4_0": (12, 128), "Q4_K": (6, 512), "Q6_K": (6, 512)}


def random_f16_scales(rng, n):
    """f16 bit patterns: magnitudes 2^-20 .. 2^-1 (normal and subnormal), either sign."""
    mag = np.exp2(rng.uniform(-20.0, -1.0, n)).astype(np.float16)
    sign = np.where(rng.random(n) < 0.25, -1.0, 1.0).astype(np.float16)
    return (mag * sign).view(np.uint16)


def raw_blocks(rng, name, rows, cols):
    tid, be, bb, f16_at = TYPES[name]
    nb = rows * cols // be
    blocks = rng.integers(0, 256, size=(nb, bb), dtype=np.uint8)
    for off in f16_at:
        bits = random_f16_scales(rng, nb)
        blocks[:, off] = (bits & 0xFF).astype(np.uint8)
        blocks[:, off + 1] = (bits >> 8).astype(np.uint8)
    return blocks.reshape(rows, cols // be * bb)


def edge_weights(rng, rows, cols):
    w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    w[0] = 0.0                                  # all-zero blocks: d = 0
    w[1] = 0.0
    w[1, 5] = 0.37                              # one spike per row
    w[2] = -1.25                                # constant negative blocks
    w[3, :32] = np.linspace(-1.0, 1.0, 32)      # evenly spaced, many ties after scaling
    w[4] = (rng.standard_normal(cols) * 3e3).astype(np.float32)  # large magnitude
    w[5, :32] = np.arange(-16, 16, dtype=np.float32) * 0.5       # exact multiples of d
    return w


def main():
    import gguf
    from gguf import GGMLQuantizationType as QT
    from gguf import quants

    out = {}
    rng = np.random.default_rng(20240611)
    for name in TYPES:
        rows, cols = RAW_SHAPE[name]
        raw = raw_blocks(rng, name, rows, cols)
        out[f"{name}_raw"] = raw
        out[f"{name}_raw_deq"] = quants.dequantize(raw, getattr(QT, name)).astype(np.float32)
        assert out[f"{name}_raw_deq"].shape == (rows, cols)
    for name in ("Q8_0", "Q4_0"):
        w = edge_weights(rng, 10, 256)
        blocks = quants.quantize(w, getattr(QT, name))
        out[f"{name}_w"] = w
        out[f"{name}_blocks"] = blocks
        out[f"{name}_deq"] = quants.dequantize(blocks, getattr(QT, name)).astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "gguf_vectors.npz"), gguf_version=np.array(gguf.__version__)
                        if hasattr(gguf, "__version__") else np.array(_version()), **out)

    path = os.path.join(HERE, "gguf_writer.gguf")
    wr = gguf.GGUFWriter(path, "llama")
    wr.add_name("fixture")
    wr.add_uint32("fixture.u32", 7)
    wr.add_int64("fixture.i64", -(2 ** 40))
    wr.add_float32("fixture.f32", 0.5)
    wr.add_bool("fixture.flag", True)
    wr.add_array("fixture.tokens", ["a", "bc", "def"])
    for name in TYPES:
        raw = out[f"{name}_raw"]
        wr.add_tensor(f"raw.{name.lower()}.weight", raw, raw_dtype=getattr(QT, name))
    wr.add_tensor("norm.weight", np.linspace(-1, 1, 24, dtype=np.float32).reshape(4, 6))
    wr.add_tensor("half.weight", np.arange(10, dtype=np.float16))
    wr.write_header_to_file()
    wr.write_kv_data_to_file()
    wr.write_tensors_to_file()
    wr.close()


def _version():
    from importlib.metadata import version
    return version("gguf")


if __name__ == "__main__":
    main()
