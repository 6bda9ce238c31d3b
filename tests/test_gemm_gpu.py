"""GPU parity of the dense matmul (j4b_matmul) against a float64 reference.

precision 1: bf16 operands on the tcgen05 tensor cores, fp32 accumulation (rel 1e-2);
precision 2: the 3-term bf16 split on the tensor cores (rel 1e-4, the fp32 tolerance);
precision 0: fp32-accurate, SIMT for small shapes and the tensor cores for large ones.
The reference CPU backend multiplies in float with an i-p-j loop (CpuBackend.java:188-216);
both are compared here with the exact product.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = {0: 1e-4, 1: 1e-2, 2: 1e-4}


def check(got, want, tol):
    got = np.asarray(got, np.float64)
    n = np.linalg.norm(want)
    assert np.linalg.norm(got - want) / n <= tol
    assert np.abs(got - want).max() <= tol * np.abs(want).max() * 4


@pytest.mark.parametrize("precision", [1, 2])
@pytest.mark.parametrize("m,k,n", [(128, 64, 128), (256, 784, 512), (300, 100, 70), (7, 5, 3),
                                   (129, 65, 257), (1024, 4096, 1024)])
def test_tensor_core_matmul(backend, m, k, n, precision):
    rng = np.random.default_rng(m * 7 + k * 3 + n)
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((k, n)).astype(np.float32)
    out = backend.matmul(backend.upload(a, a.shape), backend.upload(b, b.shape), precision)
    got = backend.download(out).reshape(m, n)
    check(got, a.astype(np.float64) @ b.astype(np.float64), TOL[precision])


@pytest.mark.parametrize("precision", [0, 1, 2])
def test_batched_matmul(backend, precision):
    rng = np.random.default_rng(11)
    a = rng.standard_normal((3, 200, 96)).astype(np.float32)
    b = rng.standard_normal((3, 96, 150)).astype(np.float32)
    out = backend.batched_matmul(backend.upload(a, a.shape), backend.upload(b, b.shape), precision)
    got = backend.download(out).reshape(3, 200, 150)
    check(got, a.astype(np.float64) @ b.astype(np.float64), TOL[precision])


def test_auto_precision_large_shape_is_fp32_accurate_and_deterministic(backend):
    rng = np.random.default_rng(5)
    a = rng.standard_normal((512, 1024)).astype(np.float32)
    b = rng.standard_normal((1024, 768)).astype(np.float32)
    A, B = backend.upload(a, a.shape), backend.upload(b, b.shape)
    g1 = backend.download(backend.matmul(A, B, 0)).reshape(512, 768)
    g2 = backend.download(backend.matmul(A, B, 0)).reshape(512, 768)
    assert np.array_equal(g1, g2)
    check(g1, a.astype(np.float64) @ b.astype(np.float64), 1e-4)
