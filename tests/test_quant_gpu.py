"""GPU parity of the quantized path (QuantizedOps) against the C oracle.

Bars (stated per test): dequantised weights and encoded blocks bit-exact; GEMV outputs within a
normwise relative error of 1e-4 of the exact (float64) product of the dequantised weights --
max|y - y_exact| / max|y_exact| <= 1e-4 -- the fp32-accumulate bar.
"""
import numpy as np
import pytest
import torch

Q4_0, Q8_0, Q4_K, Q6_K, Q2_0 = 2, 8, 12, 14, 42
TYPES = [Q8_0, Q4_0, Q4_K, Q6_K, Q2_0]
REL = 1e-4

pytestmark = pytest.mark.gpu


def make(oracle, qtype, rows, cols, seed, scale=0.02):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((rows, cols)) * scale).astype(np.float32)
    return w, oracle.quantize(qtype, w)


def normwise(y, y64):
    return float(np.abs(y.astype(np.float64) - y64).max() / max(np.abs(y64).max(), 1e-30))


# ragged shapes: rows not a multiple of the 16-row tile, columns not a multiple of the 128/1024
# column chunks, a single row, a single block
SHAPES = {
    Q8_0: [(37, 96), (1, 32), (64, 1056), (130, 2080)],
    Q4_0: [(37, 96), (1, 32), (64, 1056), (130, 2080)],
    Q4_K: [(21, 256), (1, 512), (48, 1280), (130, 2304)],
    Q6_K: [(21, 256), (1, 512), (48, 1280), (130, 2304)],
    Q2_0: [(37, 128), (1, 384), (64, 1152), (130, 2176)],
}


@pytest.mark.parametrize("qtype", TYPES)
def test_gather_row_bit_exact(backend, oracle, qtype):
    for i, (rows, cols) in enumerate(SHAPES[qtype]):
        _, blob = make(oracle, qtype, rows, cols, 100 + i)
        w = backend.upload_quantized(blob, qtype, (rows, cols))
        for r in sorted({0, rows // 2, rows - 1}):
            got = backend.download(backend.quant_gather_row(w, r))
            want = oracle.gather_row(qtype, blob, rows, cols, r)
            assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (rows, cols, r)


@pytest.mark.parametrize("qtype", TYPES)
def test_device_encoder_byte_identical(backend, oracle, qtype):
    for i, (rows, cols) in enumerate(SHAPES[qtype]):
        w, blob = make(oracle, qtype, rows, cols, 200 + i)
        dev = backend.quantize(backend.upload(w, w.shape), qtype)
        assert np.array_equal(dev.cpu().numpy(), blob), (rows, cols)


@pytest.mark.parametrize("qtype", TYPES)
@pytest.mark.parametrize("batch", [1, 3, 8, 9, 16, 21, 40, 64])
def test_matvec_within_tolerance(backend, oracle, qtype, batch):
    for i, (rows, cols) in enumerate(SHAPES[qtype]):
        _, blob = make(oracle, qtype, rows, cols, 300 + i)
        w = backend.upload_quantized(blob, qtype, (rows, cols))
        x = np.random.default_rng(i).standard_normal((batch, cols)).astype(np.float32)
        y = backend.download(backend.quant_matvec(w, backend.upload(x, x.shape)))
        y64 = oracle.quant_matvec_f64(qtype, blob, rows, cols, x)
        assert normwise(y, y64) <= REL, (rows, cols, batch, normwise(y, y64))


@pytest.mark.parametrize("qtype", [Q8_0, Q4_0, Q4_K])
@pytest.mark.parametrize("batch", [17, 33, 64])
def test_matvec_add_at_decode_batches(backend, oracle, qtype, batch):
    """17..64 rows of x with `add`: GEMV passes of 16 rows, or from 33 (Q8_0) / 49 (Q4_0, Q4_K)
    rows the fused dequant-GEMM (add applied in its epilogue or in the split-K fold); ragged rows
    and columns."""
    rows, cols = (150, 1280) if qtype == Q4_K else (150, 1120)
    _, blob = make(oracle, qtype, rows, cols, 900 + batch)
    w = backend.upload_quantized(blob, qtype, (rows, cols))
    x = np.random.default_rng(batch).standard_normal((batch, cols)).astype(np.float32)
    add = np.random.default_rng(batch + 1).standard_normal((batch, rows)).astype(np.float32)
    y64 = oracle.quant_matvec_f64(qtype, blob, rows, cols, x)
    ya = backend.download(backend.quant_matvec_add(w, backend.upload(x, x.shape),
                                                   backend.upload(add, add.shape))).reshape(batch, rows)
    assert normwise(ya - add, y64) <= REL
    # a long K range: partials of several K splits folded in split order
    rows2, cols2 = 256, 8192
    _, blob2 = make(oracle, qtype, rows2, cols2, 901)
    w2 = backend.upload_quantized(blob2, qtype, (rows2, cols2))
    x2 = np.random.default_rng(5).standard_normal((batch, cols2)).astype(np.float32)
    y2 = backend.download(backend.quant_matvec(w2, backend.upload(x2, x2.shape))).reshape(batch, rows2)
    assert normwise(y2, oracle.quant_matvec_f64(qtype, blob2, rows2, cols2, x2)) <= REL


def test_reference_shaped_call_and_add(backend, oracle):
    """Rank-1 x is the reference's quantMatvec / quantMatvecAdd (CpuBackend.java:707-736)."""
    rows, cols = 48, 512
    _, blob = make(oracle, Q4_0, rows, cols, 7)
    w = backend.upload_quantized(blob, Q4_0, (rows, cols))
    x = np.random.default_rng(1).standard_normal(cols).astype(np.float32)
    add = np.random.default_rng(2).standard_normal(rows).astype(np.float32)
    y = backend.download(backend.quant_matvec(w, backend.upload(x, (cols,))))
    assert y.shape == (rows,)
    ref = oracle.quant_matvec(Q4_0, blob, rows, cols, x)[0]  # the reference's float order
    y64 = oracle.quant_matvec_f64(Q4_0, blob, rows, cols, x)[0]
    assert normwise(y, y64) <= REL and normwise(ref, y64) <= REL
    ya = backend.download(backend.quant_matvec_add(w, backend.upload(x, (cols,)),
                                                   backend.upload(add, (rows,))))
    assert normwise(ya - add, y64) <= REL
    with pytest.raises(ValueError, match="quantMatvec shape mismatch"):
        backend.quant_matvec(w, backend.upload(np.zeros(cols - 32, np.float32), (cols - 32,)))


def test_host_buffer_call(backend, oracle):
    """j4b_quant_matvec_host (copy in, GEMV, copy out on the stream) equals the device-buffer
    call bit for bit, from pinned and from pageable host memory, and rejects bad shapes."""
    import torch
    rows, cols = 160, 4096
    _, blob = make(oracle, Q4_K, rows, cols, 13)
    w = backend.upload_quantized(blob, Q4_K, (rows, cols))
    for batch in (1, 5, 16):
        x = np.random.default_rng(batch).standard_normal((batch, cols)).astype(np.float32)
        want = backend.download(backend.quant_matvec(w, backend.upload(x, x.shape)))
        for pin in (True, False):
            xh = torch.from_numpy(x)
            yh = torch.zeros(batch * rows, dtype=torch.float32)
            if pin:
                xh, yh = xh.pin_memory(), yh.pin_memory()
            backend.quant_matvec_host(w, xh, yh)
            backend.sync()
            assert np.array_equal(yh.numpy().reshape(batch, rows), want.reshape(batch, rows))
    with pytest.raises(ValueError, match="batch 1..16"):
        backend.quant_matvec_host(w, torch.zeros(17 * cols), torch.zeros(17 * rows))
    # the recorded form replays the same call: new x values in the same buffer, new products out
    batch = 8
    xh = torch.zeros((batch, cols)).pin_memory()
    yh = torch.zeros(batch * rows).pin_memory()
    plan = backend.quant_matvec_host_plan(w, xh, yh)
    for seed in (21, 22, 23):
        x = np.random.default_rng(seed).standard_normal((batch, cols)).astype(np.float32)
        xh.copy_(torch.from_numpy(x))
        plan.run()
        backend.sync()
        want = backend.download(backend.quant_matvec(w, backend.upload(x, x.shape)))
        assert np.array_equal(yh.numpy().reshape(batch, rows), want.reshape(batch, rows))


def test_repeated_calls_are_deterministic(backend, oracle):
    """The split-K arrival counters reset themselves: back-to-back calls agree bit for bit."""
    rows, cols = 160, 4096  # 4 K ranges
    _, blob = make(oracle, Q8_0, rows, cols, 11)
    w = backend.upload_quantized(blob, Q8_0, (rows, cols))
    x = backend.upload(np.random.default_rng(3).standard_normal((8, cols)).astype(np.float32),
                       (8, cols))
    first = backend.download(backend.quant_matvec(w, x))
    for _ in range(5):
        again = backend.download(backend.quant_matvec(w, x))
        assert np.array_equal(first, again)


def test_invalid_geometry_rejected(backend, oracle):
    with pytest.raises(ValueError, match="invalid quant dimensions"):
        backend.upload_quantized(np.zeros(34, np.uint8), Q8_0, (1, 33))
    with pytest.raises(ValueError, match="bytes"):
        backend.upload_quantized(np.zeros(30, np.uint8), Q8_0, (1, 32))
    with pytest.raises(NotImplementedError):
        backend.upload_quantized(np.zeros(34, np.uint8), 41, (1, 256))


@pytest.mark.parametrize("qtype,rows,cols,batch", [
    (Q8_0, 4096, 4096, 8),
    (Q4_K, 14336, 4096, 1),    # BASELINE config 3, decode
    (Q4_K, 14336, 4096, 16),   # BASELINE config 3, batch 16
    (Q4_0, 4096, 14336, 4),    # config 5 down-projection shape
    (Q6_K, 4096, 14336, 8),    # Q6_K output/down projections of GGUF Q4_K_M files
])
def test_baseline_sizes(backend, oracle, qtype, rows, cols, batch):
    """Full BASELINE shapes: device-encoded weights, checked against the float64 oracle."""
    g = torch.Generator(device="cuda").manual_seed(rows + cols)
    wt = torch.randn(rows, cols, device="cuda", generator=g) * 0.02
    blob_dev = backend.quantize(backend.wrap(wt), qtype)
    blob = blob_dev.cpu().numpy()
    w = backend.upload_quantized(blob_dev, qtype, (rows, cols))
    x = np.random.default_rng(5).standard_normal((batch, cols)).astype(np.float32)
    y = backend.download(backend.quant_matvec(w, backend.upload(x, x.shape)))
    y64 = oracle.quant_matvec_f64(qtype, blob, rows, cols, x)
    assert normwise(y, y64) <= REL
    # dequantised rows of the full matrix stay bit-exact
    for r in (0, rows - 1):
        got = backend.download(backend.quant_gather_row(w, r))
        assert np.array_equal(got, oracle.gather_row(qtype, blob, rows, cols, r))


# ---- prefill projection: y [m, rows] = x [m, cols] . W^T on the tensor cores ----
# 3-term split: normwise 1e-4. bf16 operands: 1e-2 of the magnitude of the summed products
# (|x| . |W|^T), the scale of a bf16 rounding-error bound -- a lone output of a short dot product
# can cancel below its terms' magnitude, where a plain normwise ratio would measure cancellation.

@pytest.mark.parametrize("qtype", TYPES)
@pytest.mark.parametrize("precision,tol", [(1, 1e-2), (2, 1e-4)])
def test_quant_gemm_prefill(backend, oracle, qtype, precision, tol):
    for i, (rows, cols) in enumerate(SHAPES[qtype]):
        _, blob = make(oracle, qtype, rows, cols, 300 + i)
        w = backend.upload_quantized(blob, qtype, (rows, cols))
        deq = oracle.dequantize(qtype, blob, rows, cols).astype(np.float64)
        for m in (1, 77, 300):
            x = np.random.default_rng(m + i).standard_normal((m, cols)).astype(np.float32)
            y = backend.download(backend.quant_gemm(w, backend.upload(x, x.shape), precision)).reshape(m, rows)
            want = x.astype(np.float64) @ deq.T
            if precision == 1:
                scale = (np.abs(x).astype(np.float64) @ np.abs(deq).T).max()
                err = float(np.abs(y - want).max() / scale)
            else:
                err = normwise(y, want)
            assert err <= tol, (rows, cols, m, err)


def test_quant_gemm_config5_shape(backend, oracle):
    """A Q4_0 FFN projection at prefill scale: x [2048, 4096] . W^T, W [14336 x 4096]."""
    rows, cols, m = 14336, 4096, 2048
    g = torch.Generator(device="cuda").manual_seed(5)
    w32 = (torch.randn(rows, cols, device="cuda", generator=g) * 0.02).contiguous()
    blob = backend.quantize(backend.wrap(w32), Q4_0)
    w = backend.upload_quantized(blob, Q4_0, (rows, cols))
    x = torch.randn(m, cols, device="cuda", generator=g)
    y = backend.quant_gemm(w, backend.wrap(x), 1).tensor.reshape(m, rows)
    # expected weights from the C oracle's decode of the encoded blocks (not the engine's own gather)
    host_blob = blob.cpu().numpy()
    deq = torch.from_numpy(np.stack([oracle.gather_row(Q4_0, host_blob, rows, cols, r)
                                     for r in range(0, rows, 512)])).to(x.device)
    want = x.double() @ deq.double().T
    got = y[:, ::512].double()
    err = (got - want).abs().max() / want.abs().max()
    assert err.item() <= 1e-2
