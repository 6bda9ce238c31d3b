"""The GGUF block formats pinned to llama.cpp's own codecs (Python package `gguf` 0.19.0, whose
gguf/quants.py restates ggml's published block layouts). The reference has only the formats'
geometry (core/tensor/QuantType.java:8-10); these fixtures, made by
tests/golden/make_gguf_vectors.py, are the pin:

  CPU  the oracle's Q8_0/Q4_0 encoders are byte-identical to gguf's, and its Q8_0/Q4_0/Q4_K/Q6_K
       decoders bit-exact against gguf's on random blocks (random codes; f16 scales of either
       sign, normal and subnormal) and on edge-case weights; the engine's GGUF reader reads a file
       written by gguf.GGUFWriter, and gguf.GGUFReader reads a file the engine's writer wrote.
  GPU  quant_gather_row of the uploaded fixture blocks is bit-exact against gguf's
       dequantisation, the device encoder is byte-identical to gguf's, and the GEMV over the
       fixture blocks is within the 1e-4 normwise bar of the float64 product of gguf's
       dequantised weights.
"""
import os

import numpy as np
import pytest

from jax4j_b200 import gguf as j4b_gguf

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden")
IDS = {"Q8_0": 8, "Q4_0": 2, "Q4_K": 12, "Q6_K": 14}
ENCODED = ("Q8_0", "Q4_0")  # the types gguf 0.19 can encode


@pytest.fixture(scope="module")
def vectors():
    d = np.load(os.path.join(GOLDEN, "gguf_vectors.npz"))
    assert str(d["gguf_version"]) == "0.19.0"
    return d


def same_bits(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


@pytest.mark.parametrize("name", sorted(IDS))
def test_oracle_decoder_matches_gguf(oracle, vectors, name):
    raw, want = vectors[f"{name}_raw"], vectors[f"{name}_raw_deq"]
    rows, cols = want.shape
    assert same_bits(oracle.dequantize(IDS[name], raw.reshape(-1), rows, cols), want)
    if name in ENCODED:
        blocks, deq = vectors[f"{name}_blocks"], vectors[f"{name}_deq"]
        assert same_bits(oracle.dequantize(IDS[name], blocks.reshape(-1), *deq.shape), deq)


@pytest.mark.parametrize("name", ENCODED)
def test_oracle_encoder_matches_gguf(oracle, vectors, name):
    w = vectors[f"{name}_w"]
    assert np.array_equal(oracle.quantize(IDS[name], w), vectors[f"{name}_blocks"].reshape(-1))


def test_reader_reads_a_gguf_writer_file(vectors):
    f = j4b_gguf.read(os.path.join(GOLDEN, "gguf_writer.gguf"))
    assert f.version == 3
    assert f.metadata["general.architecture"] == "llama" and f.metadata["general.name"] == "fixture"
    assert f.metadata["fixture.u32"] == 7 and f.metadata["fixture.i64"] == -(2 ** 40)
    assert f.metadata["fixture.f32"] == 0.5 and f.metadata["fixture.flag"] is True
    assert f.metadata["fixture.tokens"] == ["a", "bc", "def"]
    for name, tid in IDS.items():
        t = f.tensor(f"raw.{name.lower()}.weight")
        assert t.type_id == tid and t.shape == vectors[f"{name}_raw_deq"].shape
        assert np.array_equal(np.asarray(f.data(t.name)), vectors[f"{name}_raw"].reshape(-1))
    norm = f.tensor("norm.weight")
    assert norm.type_id == 0 and norm.shape == (4, 6)
    assert np.array_equal(np.asarray(f.data("norm.weight")).view(np.float32),
                          np.linspace(-1, 1, 24, dtype=np.float32))
    half = f.tensor("half.weight")
    assert half.type_id == 1 and half.shape == (10,)
    assert np.array_equal(np.asarray(f.data("half.weight")).view(np.float16), np.arange(10, dtype=np.float16))


def test_gguf_reader_reads_our_file(tmp_path, vectors):
    gg = pytest.importorskip("gguf")
    path = str(tmp_path / "ours.gguf")
    tensors = [(f"raw.{n.lower()}", vectors[f"{n}_raw_deq"].shape, IDS[n], vectors[f"{n}_raw"].reshape(-1))
               for n in sorted(IDS)]
    j4b_gguf.write(path, {"general.architecture": "llama", "n": 3}, tensors)
    r = gg.GGUFReader(path)
    by_name = {t.name: t for t in r.tensors}
    for name, shape, tid, raw in tensors:
        t = by_name[name]
        assert int(t.tensor_type) == tid
        assert tuple(int(v) for v in reversed(t.shape)) == shape
        assert np.array_equal(np.asarray(t.data).reshape(-1).view(np.uint8), raw)
        deq = gg.quants.dequantize(np.asarray(t.data), t.tensor_type)
        assert same_bits(deq.reshape(shape), vectors[f"{name[4:].upper()}_raw_deq"])


# ---- the engine on the GPU ----

@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(IDS))
def test_engine_gather_row_matches_gguf(backend, vectors, name):
    raw, want = vectors[f"{name}_raw"], vectors[f"{name}_raw_deq"]
    rows, cols = want.shape
    w = backend.upload_quantized(raw.reshape(-1), IDS[name], (rows, cols))
    for r in range(rows):
        assert same_bits(backend.download(backend.quant_gather_row(w, r)), want[r]), r


@pytest.mark.gpu
@pytest.mark.parametrize("name", ENCODED)
def test_engine_encoder_matches_gguf(backend, vectors, name):
    w = vectors[f"{name}_w"]
    blob = backend.quantize(backend.upload(w, w.shape), IDS[name])
    assert np.array_equal(blob.cpu().numpy(), vectors[f"{name}_blocks"].reshape(-1))


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(IDS))
@pytest.mark.parametrize("batch", [1, 8, 16])
def test_engine_gemv_on_gguf_blocks(backend, vectors, name, batch):
    """Normwise relative error <= 1e-4 against the float64 product of gguf's dequantised rows."""
    raw, deq = vectors[f"{name}_raw"], vectors[f"{name}_raw_deq"]
    rows, cols = deq.shape
    w = backend.upload_quantized(raw.reshape(-1), IDS[name], (rows, cols))
    x = np.random.default_rng(batch).standard_normal((batch, cols)).astype(np.float32)
    y = backend.download(backend.quant_matvec(w, backend.upload(x, x.shape))).reshape(batch, rows)
    y64 = x.astype(np.float64) @ deq.astype(np.float64).T
    assert np.abs(y - y64).max() / np.abs(y64).max() <= 1e-4
