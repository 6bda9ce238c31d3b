"""2-D convolution (ComputeBackend.conv2d / conv2dGradInput / conv2dGradWeight) and its AD and
vmap rules. The oracle restates CpuBackend.java:479-609 and is pinned here against an
independent numpy convolution and the reference's TransformsTest known answers
(mappedConvolutionAndDerivatives; the vmapped conv2dGradWeight of
structuredGradientsAndRuleContracts' neighbour test). The engine (im2col + tensor-core GEMM) is
checked against the oracle: fp32-accurate mode normwise 1e-4, bf16 operands 1e-2 (marked gpu).
"""
import numpy as np
import pytest

from jax4j_b200 import transforms as T
from jax4j_b200 import vmap as V
from jax4j_b200.tensor import ConvSpec, Tensor

SPECS = [  # (batch, spec)
    (2, ConvSpec(1, 2, 2, 1, 1, 1, 0)),
    (3, ConvSpec(3, 8, 7, 4, 3, 1, 1)),
    (2, ConvSpec(4, 9, 9, 6, 3, 2, 0)),
    (1, ConvSpec(2, 6, 5, 3, 5, 1, 2)),
    (4, ConvSpec(8, 16, 16, 16, 3, 2, 1)),
    (8, ConvSpec(32, 32, 32, 64, 3, 1, 1)),  # large enough for the tensor-core forward at fp32 accuracy
]


def numpy_conv(x, w, spec: ConvSpec):
    """Direct correlation over the zero-padded image (an independent formulation)."""
    b = x.shape[0]
    img = x.reshape(b, spec.in_channels, spec.in_height, spec.in_width).astype(np.float64)
    img = np.pad(img, ((0, 0), (0, 0), (spec.pad, spec.pad), (spec.pad, spec.pad)))
    ker = w.reshape(spec.out_channels, spec.in_channels, spec.kernel, spec.kernel).astype(np.float64)
    out = np.zeros((b, spec.out_channels, spec.out_height, spec.out_width))
    for oh in range(spec.out_height):
        for ow in range(spec.out_width):
            win = img[:, :, oh * spec.stride:oh * spec.stride + spec.kernel, ow * spec.stride:ow * spec.stride + spec.kernel]
            out[:, :, oh, ow] = np.einsum("bckl,ockl->bo", win, ker)
    return out.reshape(b, -1)


def rand(shape, seed):
    return np.random.default_rng(seed).standard_normal(shape).astype(np.float32)


def normwise(a, b):
    return float(np.abs(np.asarray(a, np.float64) - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.mark.parametrize("batch,spec", SPECS)
def test_oracle_against_numpy(oracle, batch, spec):
    x, w = rand((batch, spec.input_size), 1), rand(spec.weight_shape(), 2)
    y = numpy_conv(x, w, spec)
    assert normwise(oracle.conv2d(x, w, spec.ints()), y) < 1e-6
    # the gradients are the adjoints of the forward map: <conv(x, w), u> = <x, dX(u)> = <w, dW(u)>
    u = rand((batch, spec.output_size), 3)
    lhs = float(np.sum(y * u))
    dx = oracle.conv2d_grad_input(u, w, spec.ints())
    dw = oracle.conv2d_grad_weight(x, u, spec.ints())
    assert abs(float(np.sum(x.astype(np.float64) * dx)) - lhs) <= 1e-4 * max(1.0, abs(lhs))
    assert abs(float(np.sum(w.astype(np.float64) * dw)) - lhs) <= 1e-4 * max(1.0, abs(lhs))


def test_spec_validation():
    with pytest.raises(ValueError, match="does not fit"):
        ConvSpec(1, 2, 2, 1, 5, 1, 0)
    with pytest.raises(ValueError, match="positive"):
        ConvSpec(0, 2, 2, 1, 1, 1, 0)
    s = ConvSpec(3, 32, 32, 8, 3, 2, 1)
    assert (s.out_height, s.out_width, s.weight_shape(), s.next(16, 3, 1, 1).in_channels) == (16, 16, (8, 27), 8)


@pytest.fixture(params=["oracle", pytest.param("b200", marks=pytest.mark.gpu)])
def be(request, oracle):
    if request.param == "oracle":
        from oracle.backend import OracleBackend
        return OracleBackend()
    from jax4j_b200.backend import B200Backend
    return B200Backend(0)


def arr(be, a):
    a = np.asarray(a, np.float32)
    return Tensor(be, be.upload(a, a.shape))


def get(t):
    return np.asarray(t.backend.download(t.buffer))


def test_mapped_convolution_and_derivatives(be):
    """TransformsTest.mappedConvolutionAndDerivatives and the vmapped conv2dGradWeight case."""
    spec = ConvSpec(1, 2, 2, 1, 1, 1, 0)
    x = arr(be, np.arange(1, 9).reshape(2, 1, 4))
    w = arr(be, [2, 3]).reshape(2, 1, 1)
    out = V.apply_tree(lambda ts: ts[0].conv2d(ts[1], spec), [x, w], [0, 0], [0])
    np.testing.assert_allclose(get(out).reshape(-1), [2, 4, 6, 8, 15, 18, 21, 24], atol=1e-5)
    w1 = arr(be, [2]).reshape(1, 1)
    dx = V.apply_tree(lambda ts: T.grad(lambda t: t.conv2d(ts[1], spec).sum(), ts[0]), [x, w1], [0, None], [0])
    np.testing.assert_allclose(get(dx).reshape(-1), [2] * 8, atol=1e-5)
    up = arr(be, [1, 1, 1, 1]).reshape(1, 4)
    dw = V.apply_tree(lambda ts: ts[0].conv2d_grad_weight(ts[1], spec), [x, up], [0, None], [0])
    np.testing.assert_allclose(get(dw).reshape(-1), [10, 26], atol=0)


def test_gradients_of_a_loss_through_conv(be, oracle):
    batch, spec = 3, ConvSpec(2, 7, 6, 3, 3, 1, 1)
    xh, wh = rand((batch, spec.input_size), 11), rand(spec.weight_shape(), 12)
    x, w = arr(be, xh), arr(be, wh)
    gx = T.grad(lambda t: t.conv2d(w, spec).tanh().sum(), x)
    gw = T.grad(lambda t: x.conv2d(t, spec).tanh().sum(), w)
    y = oracle.conv2d(xh, wh, spec.ints())
    up = (1 - np.tanh(y.astype(np.float64)) ** 2).astype(np.float32)
    assert normwise(get(gx), oracle.conv2d_grad_input(up, wh, spec.ints()).astype(np.float64)) < 1e-4
    assert normwise(get(gw), oracle.conv2d_grad_weight(xh, up, spec.ints()).astype(np.float64)) < 1e-4


@pytest.mark.gpu
@pytest.mark.parametrize("batch,spec", SPECS)
@pytest.mark.parametrize("precision,tol", [(0, 1e-4), (1, 1e-2)])
def test_engine_matches_the_oracle(backend, oracle, batch, spec, precision, tol):
    x, w, u = rand((batch, spec.input_size), 21), rand(spec.weight_shape(), 22), rand((batch, spec.output_size), 23)
    dx_, dw_, du = (backend.upload(a, a.shape) for a in (x, w, u))
    y = backend.download(backend.conv2d(dx_, dw_, spec, precision))
    assert normwise(y, oracle.conv2d(x, w, spec.ints()).astype(np.float64)) <= tol
    gi = backend.download(backend.conv2d_grad_input(du, dw_, spec, precision))
    assert normwise(gi, oracle.conv2d_grad_input(u, w, spec.ints()).astype(np.float64)) <= tol
    gw = backend.download(backend.conv2d_grad_weight(dx_, du, spec, precision))
    assert normwise(gw, oracle.conv2d_grad_weight(x, u, spec.ints()).astype(np.float64)) <= tol


@pytest.mark.gpu
def test_engine_rejects_bad_shapes(backend):
    spec = ConvSpec(2, 4, 4, 3, 3, 1, 0)
    x = backend.upload(np.zeros((2, 30), np.float32), (2, 30))
    w = backend.upload(np.zeros(spec.weight_shape(), np.float32), spec.weight_shape())
    with pytest.raises(ValueError, match="do not match"):
        backend.conv2d(x, w, spec)


@pytest.mark.gpu
def test_tensor_core_matmul_into_an_unaligned_output(backend):
    """The tensor-core GEMM stores C with 16-byte vector stores only where C is 16-byte aligned;
    an output that starts one float into a buffer (a conv scratch sub-buffer, a caller's slice)
    takes the scalar store path."""
    from jax4j_b200 import _lib
    m, k, n = 9, 27, 40
    a, b = rand((m, k), 31), rand((k, n), 32)
    da, db = backend.upload(a, a.shape), backend.upload(b, b.shape)
    out = backend.upload(np.zeros(m * n + 1, np.float32), (m * n + 1,))
    _lib.call("j4b_matmul", da.ptr, db.ptr, out.ptr + 4, 1, m, k, n, 1, backend.stream)
    got = backend.download(out)[1:].reshape(m, n)
    assert normwise(got, a.astype(np.float64) @ b) <= 1e-2
