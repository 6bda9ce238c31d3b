"""GPU parity of the eager SPI primitives against the oracle (CpuBackend semantics).

Bars: IEEE-exact ops (add/sub/mul/div/max/min/neg/abs/sign/relu/sqrt, transpose, broadcast,
reindex, uniforms, argmax, maxAxis, maxAxisBackward, fill) bit-exact; library transcendentals
within 4e-6 relative per element; sums and matmul within 1e-5 / 1e-4 normwise relative.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

EXACT_UNARY = ["NEG", "SQRT", "RELU", "ABS", "SIGN"]
APPROX_UNARY = ["EXP", "LOG", "RSQRT", "TANH", "SIGMOID"]


def rng(seed=0):
    return np.random.default_rng(seed)


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def same(a, b):
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    nan = np.isnan(a) & np.isnan(b)
    return np.array_equal(bits(a)[~nan], bits(b)[~nan]) and np.array_equal(np.isnan(a), np.isnan(b))


def special_values(n, seed=0):
    x = rng(seed).standard_normal(n).astype(np.float32) * 3
    x[:8] = [0.0, -0.0, np.nan, np.inf, -np.inf, 1.0, -1.0, 1e-40]
    return x


@pytest.mark.parametrize("op", ["ADD", "SUB", "MUL", "DIV", "MAX", "MIN"])
def test_binary_and_scalar_bit_exact(backend, oracle, op):
    a = special_values(1003, 1)
    b = special_values(1003, 2)
    b[:8] = [-0.0, 0.0, 1.0, np.nan, 2.0, -np.inf, 0.0, -0.0]
    got = backend.download(backend.binary(op, backend.upload(a, a.shape), backend.upload(b, b.shape)))
    assert same(got, oracle.binary(op, a, b))
    for v in (2.5, -0.0, 1e-3):
        got = backend.download(backend.scalar(op, backend.upload(a, a.shape), v))
        assert same(got, oracle.scalar(op, a, v))


@pytest.mark.parametrize("op", EXACT_UNARY + APPROX_UNARY)
def test_unary(backend, oracle, op):
    a = special_values(4096, 3)
    if op in ("LOG", "SQRT", "RSQRT"):
        a = np.abs(a)
    got = backend.download(backend.unary(op, backend.upload(a, a.shape)))
    want = oracle.unary(op, a)
    if op in EXACT_UNARY:
        assert same(got, want)
    else:
        finite = np.isfinite(want) & (np.abs(want) > 1e-30)
        assert np.array_equal(np.isnan(got), np.isnan(want))
        rel = np.abs(got[finite] - want[finite]) / np.abs(want[finite])
        assert rel.max() <= 4e-6, (op, rel.max())


def test_fill_transpose_broadcast(backend, oracle):
    f = backend.download(backend.full(-2.5, (3,)))  # CudaTensorTest.java:35-40
    assert np.array_equal(f, np.float32([-2.5, -2.5, -2.5]))
    for r, c in [(1, 1), (33, 65), (256, 10), (784, 512)]:
        a = rng(r).standard_normal((r, c)).astype(np.float32)
        got = backend.download(backend.transpose(backend.upload(a, a.shape)))
        assert np.array_equal(got, oracle.transpose(a))
    a = np.arange(6, dtype=np.float32).reshape(2, 1, 3)
    got = backend.download(backend.broadcast_to(backend.upload(a, a.shape), (4, 2, 5, 3)))
    assert np.array_equal(got, oracle.broadcast_to(a, (4, 2, 5, 3)))
    g = np.float32([1.0, 2.0])
    got = backend.download(backend.broadcast_to(backend.upload(g, (2,)), (3, 2)))
    assert np.array_equal(got, np.broadcast_to(g, (3, 2)))


def test_matmul_kat_and_random(backend, oracle):
    a = np.float32([[1, 2, 3], [4, 5, 6]])
    b = np.float32([[7, 8], [9, 10], [11, 12]])
    c = backend.download(backend.matmul(backend.upload(a, a.shape), backend.upload(b, b.shape)))
    assert np.array_equal(c, np.float32([[58, 64], [139, 154]]))  # CudaTensorTest.java:27-33
    # the MLP's shapes, including the skinny ones (n = 10: the logits layer and its weight
    # gradient; k = 10: the gradient into the hidden layer), and ragged small ones
    for (m, k, n) in [(256, 784, 512), (256, 512, 10), (512, 256, 10), (256, 10, 512), (784, 256, 512),
                      (5, 7, 3), (33, 100, 32), (1, 1000, 1), (70, 33, 65)]:
        a = rng(m).standard_normal((m, k)).astype(np.float32)
        b = rng(n).standard_normal((k, n)).astype(np.float32)
        got = backend.download(backend.matmul(backend.upload(a, a.shape), backend.upload(b, b.shape)))
        want = a.astype(np.float64) @ b.astype(np.float64)
        assert np.abs(got - want).max() / np.abs(want).max() <= 1e-4
    for (bt, m, k, n) in [(3, 4, 5, 6), (2, 40, 300, 7)]:
        a = rng(m).standard_normal((bt, m, k)).astype(np.float32)
        b = rng(n).standard_normal((bt, k, n)).astype(np.float32)
        got = backend.download(backend.batched_matmul(backend.upload(a, a.shape), backend.upload(b, b.shape)))
        np.testing.assert_allclose(got, oracle.batched_matmul(a, b), rtol=1e-4, atol=1e-4)
    a = rng(9).standard_normal((3, 4, 5)).astype(np.float32)
    b = rng(8).standard_normal((3, 5, 6)).astype(np.float32)
    got = backend.download(backend.batched_matmul(backend.upload(a, a.shape),
                                                  backend.upload(b, b.shape)))
    np.testing.assert_allclose(got, oracle.batched_matmul(a, b), rtol=1e-5, atol=1e-5)


def test_full_reductions(backend, oracle):
    for n in (1, 1000, 1 << 20, 3_000_017):
        a = rng(n).standard_normal(n).astype(np.float32)
        s = backend.download(backend.reduce_sum(backend.upload(a, (n,))))
        assert abs(float(s[0]) - float(oracle.reduce_sum(a)[0])) <= 1e-6 * max(1.0, np.abs(a).sum())
        m = backend.download(backend.reduce_max(backend.upload(a, (n,))))
        assert m[0] == oracle.reduce_max(a)[0]
    a = np.float32([np.nan, -1.0, 3.0, np.nan])  # reduceMax skips NaN (strict >)
    assert backend.download(backend.reduce_max(backend.upload(a, (4,))))[0] == 3.0


@pytest.mark.parametrize("shape,axis", [((4096, 8192), 1), ((256, 10), 1), ((4096, 8192), 0),
                                        ((256, 512), 0), ((3, 5, 7), 1), ((2, 1, 9), 2)])
def test_axis_reductions(backend, oracle, shape, axis):
    a = rng(sum(shape)).standard_normal(shape).astype(np.float32)
    a.reshape(-1)[::97] = 0.5  # ties
    buf = backend.upload(a, shape)
    s = backend.download(backend.sum_axis(buf, axis, True))
    want = oracle.sum_axis(a, axis, True)
    assert np.abs(s - want).max() <= 1e-6 * max(1.0, np.abs(a).sum(axis=axis).max())
    assert same(backend.download(backend.max_axis(buf, axis)), oracle.max_axis(a, axis))
    assert same(backend.download(backend.arg_max_axis(buf, axis)), oracle.argmax_axis(a, axis))
    up = rng(1).standard_normal(oracle.max_axis(a, axis).shape).astype(np.float32)
    got = backend.download(backend.max_axis_backward(backend.upload(up, up.shape), buf, axis))
    assert same(got, oracle.max_axis_backward(up, a, axis))


def test_axis_nan_rules(backend, oracle):
    a = np.float32([[1, np.nan, 3, np.nan], [2, 5, 5, -1], [-np.inf, -np.inf, -np.inf, -np.inf]])
    for axis in (0, 1):
        buf = backend.upload(a, a.shape)
        assert same(backend.download(backend.max_axis(buf, axis)), oracle.max_axis(a, axis))
        assert same(backend.download(backend.arg_max_axis(buf, axis)), oracle.argmax_axis(a, axis))


def test_reindex_scatter(backend, oracle):
    a = rng(4).standard_normal(1000).astype(np.float32)
    m = rng(5).integers(-1, 1000, 3000).astype(np.int32)
    got = backend.download(backend.reindex(backend.upload(a, (1000,)), (3000,), m))
    assert same(got, oracle.reindex(a, (3000,), m))
    u = rng(6).standard_normal(3000).astype(np.float32)
    got = backend.download(backend.scatter_add(backend.upload(u, (3000,)), (1000,), m))
    np.testing.assert_allclose(got, oracle.scatter_add(u, (1000,), m), rtol=1e-5, atol=1e-5)
    with pytest.raises(ValueError, match="index out of bounds"):
        backend.reindex(backend.upload(a, (1000,)), (1,), [1000])


def test_random_streams(backend, oracle):
    u = backend.download(backend.random_uniform(123, 7, (100_003,)))
    assert np.array_equal(u, oracle.random_uniform(123, 7, 100_003))  # bit-exact
    z = backend.download(backend.random_normal(0, 0, (100_003,)))
    np.testing.assert_allclose(z, oracle.random_normal(0, 0, 100_003), rtol=2e-6, atol=2e-6)


def test_shape_ops(backend, oracle):
    a = rng(7).standard_normal((4, 3, 2)).astype(np.float32)
    buf = backend.upload(a, a.shape)
    assert np.array_equal(backend.download(backend.slice_axis0(buf, 2)), a[2])
    st = backend.stack_axis0([backend.upload(a[i], a[i].shape) for i in range(4)])
    assert np.array_equal(backend.download(st), a)
    assert np.array_equal(backend.download(backend.reshape(buf, (6, 4))), a.reshape(6, 4))
    with pytest.raises(ValueError, match="out of bounds"):
        backend.slice_axis0(buf, 4)
    r = rng(8).standard_normal(100).astype(np.float32)
    up = rng(9).standard_normal(100).astype(np.float32)
    got = backend.download(backend.relu_backward(backend.upload(up, (100,)), backend.upload(r, (100,))))
    assert np.array_equal(got, oracle.relu_backward(up, r))
