"""GGUF container: write / read round trips of metadata and tensor data, the format's size and
alignment rules (QuantType.byteSizeFor, QuantType.java:46-53), and malformed files. The GPU test
uploads a file's quantised matrices and checks their dequantised rows against the oracle."""
import struct

import numpy as np
import pytest

from jax4j_b200 import gguf


def _blobs(oracle):
    rng = np.random.default_rng(4)
    w4 = (rng.standard_normal((48, 256)) * 0.02).astype(np.float32)
    w8 = (rng.standard_normal((16, 128)) * 0.02).astype(np.float32)
    wk = (rng.standard_normal((8, 512)) * 0.02).astype(np.float32)
    w6 = (rng.standard_normal((24, 256)) * 0.02).astype(np.float32)
    f = rng.standard_normal((3, 5)).astype(np.float32)
    return [("blk.0.attn_q.weight", (48, 256), 2, oracle.quantize(2, w4)),
            ("blk.0.ffn_up.weight", (16, 128), 8, oracle.quantize(8, w8)),
            ("blk.0.ffn_down.weight", (8, 512), 12, oracle.quantize(12, wk)),
            ("output.weight", (24, 256), 14, oracle.quantize(14, w6)),
            ("token_norm", (3, 5), 0, f.view(np.uint8)),
            ("scale", (7,), 1, np.arange(7, dtype=np.float16).view(np.uint8))]


META = {"general.architecture": "llama", "general.name": "tiny", "llama.block_count": 1,
        "llama.rope.freq_base": 10000.0, "tokenizer.ggml.tokens": ["a", "b", "c"],
        "flags": [1, 2, 3], "big": 2 ** 40, "neg": -5, "ok": True}


@pytest.mark.parametrize("alignment", [32, 64])
def test_round_trip(tmp_path, oracle, alignment):
    path = str(tmp_path / "m.gguf")
    tensors = _blobs(oracle)
    gguf.write(path, META, tensors, alignment=alignment)
    f = gguf.read(path)
    assert f.version == 3 and f.alignment == alignment and f.data_offset % alignment == 0
    for k, v in META.items():
        assert f.metadata[k] == (pytest.approx(v) if isinstance(v, float) else v)
    assert [t.name for t in f.tensors] == [t[0] for t in tensors]
    for name, shape, tid, raw in tensors:
        t = f.tensor(name)
        assert t.shape == shape and t.type_id == tid and t.offset % alignment == 0
        assert t.nbytes == gguf.byte_size(tid, int(np.prod(shape)))
        assert np.array_equal(np.asarray(f.data(name)), np.asarray(raw, np.uint8).reshape(-1))


def test_size_rules_and_malformed_files(tmp_path, oracle):
    assert gguf.byte_size(14, 512) == 420 and gguf.byte_size(2, 64) == 36
    with pytest.raises(ValueError, match="not block-aligned"):
        gguf.byte_size(12, 100)
    with pytest.raises(ValueError, match="unknown ggml quant type id"):
        gguf.byte_size(99, 32)
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGML" + bytes(40))
    with pytest.raises(ValueError, match="not a GGUF file"):
        gguf.read(str(bad))
    path = str(tmp_path / "m.gguf")
    gguf.write(path, META, _blobs(oracle))
    raw = open(path, "rb").read()
    (tmp_path / "v9.gguf").write_bytes(raw[:4] + struct.pack("<I", 9) + raw[8:])
    with pytest.raises(ValueError, match="unsupported GGUF version"):
        gguf.read(str(tmp_path / "v9.gguf"))
    (tmp_path / "cut.gguf").write_bytes(raw[:60])
    with pytest.raises(ValueError, match="truncated"):
        gguf.read(str(tmp_path / "cut.gguf"))
    with pytest.raises(ValueError, match="bytes for shape"):
        gguf.write(str(tmp_path / "x.gguf"), {}, [("w", (2, 32), 2, np.zeros(10, np.uint8))])


@pytest.mark.gpu
def test_load_quantized_matrices_match_the_oracle(tmp_path, oracle, backend):
    path = str(tmp_path / "m.gguf")
    tensors = _blobs(oracle)
    gguf.write(path, META, tensors)
    f = gguf.read(path)
    loaded = gguf.load_quantized(backend, f)
    for name, shape, tid, raw in tensors:
        buf = loaded[name]
        if tid in (0, 1):
            want = np.asarray(raw).reshape(-1).view(np.float32 if tid == 0 else np.float16).astype(np.float32)
            assert np.array_equal(backend.download(buf).reshape(-1), want)
            continue
        assert buf.shape == shape
        for r in (0, shape[0] - 1):
            got = backend.download(backend.quant_gather_row(buf, r))
            assert np.array_equal(got, oracle.gather_row(tid, np.asarray(raw), shape[0], shape[1], r))
