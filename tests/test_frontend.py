"""CPU tests of the front end (Tensor / Transforms / Vmap / Jit tracing) and of the tape planner.

The front end runs here on the oracle backend (oracle/backend.py) and is pinned to the JAX
fixtures the reference's own tests load: JaxParityTest.java:15-38 (compiled valueAndGrad,
2e-6), VmapTest.java:10-19 (vmap of a reduction and of a gradient) and TransformsTest.java:
455-490 (three compiled Adam steps, 3e-6). Recorded tapes are replayed by the oracle's tape
interpreter and must equal eager execution exactly. The engine's tape compiler is exercised
without a device through j4b_tape_dryrun: planning, code generation and NVRTC compilation.
"""
import numpy as np
import pytest

from jax4j_b200 import jit as J
from jax4j_b200 import nn
from jax4j_b200 import transforms as T
from jax4j_b200 import vmap as V
from jax4j_b200.tensor import Tensor


def f32(x):
    return np.asarray(x, np.float32)


@pytest.fixture(scope="module")
def be(oracle):
    from oracle.backend import OracleBackend
    return OracleBackend()


def tensor(be, x):
    return Tensor(be, be.upload(f32(x)))


def get(t):
    return t.backend.download(t.buffer)


def test_compiled_value_and_grad_matches_jax(be, golden):
    def body(x):
        def f(v):
            y = v.mul(1.5).tanh()
            return y.mul(y).sum()
        value, grad = T.value_and_grad(f, x)
        return [value, grad]

    compiled = J.compile(body)
    value, grad = compiled(tensor(be, golden["input"]))
    np.testing.assert_allclose(get(value), golden["value"], atol=2e-6, rtol=0)
    np.testing.assert_allclose(get(grad), golden["gradient"], atol=2e-6, rtol=0)
    value, grad = compiled(tensor(be, [0, 0, 0, 0]))
    assert abs(get(value)[0]) <= 1e-6 and np.all(np.abs(get(grad)) <= 1e-6)
    assert compiled.traces == 1 and compiled.cached_plan_count() == 1


def test_vmap_reduction_and_gradient(be, golden):
    x = tensor(be, [[1, 2, 3], [4, 5, 6]])
    out = J.compile(lambda t: V.apply(lambda r: r.mul(r).sum(), t))(x)
    assert out.shape == (2, 1)
    np.testing.assert_allclose(get(out).reshape(-1), [14, 77], atol=1e-6)
    grads = J.compile(lambda t: V.apply(lambda r: T.grad(lambda v: v.mul(v).sum(), r), t))(x)
    np.testing.assert_allclose(get(grads).reshape(-1), golden["mappedGradient"], atol=1e-6)


def test_compiled_adam_training_step(be, golden):
    opt = nn.FunctionalAdam(.01)

    def train(p, m, v, step):
        _, (g,) = T.value_and_grad_tree(lambda ps: ps[0].mul(ps[0]).sum(), [p])
        (p2,), ((m2,), (v2,), step2) = opt.update([p], [g], ([m], [v], step))
        return [p2, m2, v2, step2]

    compiled = J.compile(train)
    p = tensor(be, [1, 2])
    (m,), (v,), step = opt.initialize([p])
    for _ in range(3):
        p, m, v, step = compiled(p, m, v, step)
    assert compiled.traces == 1
    assert get(step)[0] == 3
    np.testing.assert_allclose(get(p), golden["adamParameters"], atol=3e-6, rtol=0)


def _eager_vs_tape(be, fn, inputs):
    from oracle.backend import run_tape
    eager = fn(*[tensor(be, x) for x in inputs])
    tape = J.trace(fn, [x.shape for x in inputs])
    got = run_tape(tape, inputs)
    eager = eager if isinstance(eager, list) else [eager]
    assert len(got) == len(eager)
    for e, g in zip(eager, got):
        np.testing.assert_array_equal(get(e).reshape(-1), g.reshape(-1))
    return tape


def test_rms_swiglu_tape_replays_eager(be):
    rng = np.random.default_rng(0)
    x = rng.standard_normal((8, 32)).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(32)).astype(np.float32)
    tape = _eager_vs_tape(be, nn.rms_swiglu_value_and_grad, [x, g])
    assert [tape.shapes[o] for o in tape.outputs] == [(1,), (8, 32), (32,)]


def test_rms_swiglu_gradient_matches_finite_differences(be):
    rng = np.random.default_rng(1)
    x = rng.standard_normal((3, 8)).astype(np.float64)
    g = (1 + 0.1 * rng.standard_normal(8)).astype(np.float64)

    def loss(x, g):
        h = x / np.sqrt((x * x).mean(axis=1, keepdims=True) + 1e-5) * g
        a, b = h[:, :4], h[:, 4:]
        y = a / (1 + np.exp(-a)) * b
        return (y * y).mean()

    value, dx, dg = nn.rms_swiglu_value_and_grad(tensor(be, x), tensor(be, g))
    assert abs(get(value)[0] - loss(x, g)) < 1e-5
    eps = 1e-6
    for i in range(x.size):
        d = np.zeros_like(x)
        d.flat[i] = eps
        fd = (loss(x + d, g) - loss(x - d, g)) / (2 * eps)
        assert abs(get(dx).flat[i] - fd) < 1e-4
    for i in range(g.size):
        d = np.zeros_like(g)
        d[i] = eps
        fd = (loss(x, g + d) - loss(x, g - d)) / (2 * eps)
        assert abs(get(dg)[i] - fd) < 1e-4


def test_mlp_tape_replays_eager(be):
    rng = np.random.default_rng(2)
    x = rng.standard_normal((6, 12)).astype(np.float32)
    w1 = rng.uniform(-.5, .5, (12, 8)).astype(np.float32)
    w2 = rng.uniform(-.5, .5, (8, 10)).astype(np.float32)
    b1, b2 = np.zeros(8, np.float32), np.zeros(10, np.float32)
    onehot = np.eye(10, dtype=np.float32)[rng.integers(0, 10, 6)]
    _eager_vs_tape(be, nn.mlp_value_and_grad, [w1, b1, w2, b2, x, onehot])


# ---- the engine's planner and code generator, without a device ----

def _lib():
    from jax4j_b200 import _lib as L
    try:
        L.load()
    except (RuntimeError, OSError) as e:  # pragma: no cover - build() runs before the suite
        pytest.fail(f"engine library not built: {e}")
    return L


def test_tape_plan_rms_swiglu_is_one_fused_kernel():
    L = _lib()
    tape = J.trace(nn.rms_swiglu_value_and_grad, [(4096, 8192), (8192,)])
    stats, src = L.tape_dryrun(tape.serialize())
    # forward + backward of the vmapped body: one row program plus one cross-row fold
    assert stats["groups"] == 1 and stats["folds"] == 1 and stats["eager_steps"] == 0
    assert "block_sum<512>" in src and "__ldg(reinterpret_cast<const float4*>" in src
    # the two row sums (mean square forward, its cotangent backward) reduce in float; the loss
    # keeps the double block sum
    assert src.count("block_sumf<512>(") == 2
    # the backward reuses the forward's per-row rsqrt (one call besides the helper's definition)
    assert src.count("jrsqrt(") == 2
    # dg's per-CTA partial is stored on its first flush: no zeroing pass, no read-back
    assert "col_first" in src and "+ j] = 0.0;" not in src


def test_tape_plan_mlp_and_adam():
    L = _lib()
    shapes = [(784, 512), (512,), (512, 10), (10,), (256, 784), (256, 10)]
    tape = J.trace(nn.mlp_value_and_grad, shapes)
    stats, _ = L.tape_dryrun(tape.serialize())
    # forward 2, backward 4 (the cotangent of the constant x is recorded but never read)
    matmuls = sum(c.op == "matmul" for c in tape.calls)
    assert matmuls == 6
    assert stats["eager_steps"] >= matmuls - 1 and stats["groups"] >= 2
    opt = nn.FunctionalAdam(1e-3)
    pshapes = shapes[:4]
    n = len(pshapes)
    tape = J.trace(opt._step_flat, pshapes * 4 + [(1,)])
    stats, _ = L.tape_dryrun(tape.serialize())
    assert stats["eager_steps"] == 0 and stats["groups"] <= 2, stats


def test_tape_validation_rejects_malformed_tapes():
    L = _lib()
    tape = J.trace(lambda a, b: a.matmul(b), [(2, 3), (3, 4)])
    words = tape.serialize()
    L.tape_dryrun(words)
    with pytest.raises(ValueError):
        L.tape_dryrun(words[:-1])
    bad = words.copy()
    bad[0] ^= 1
    with pytest.raises(ValueError):
        L.tape_dryrun(bad)
    bad_shape = J.trace(lambda a, b: a.matmul(b), [(2, 3), (3, 4)])
    bad_shape.shapes[bad_shape.inputs[1]] = (5, 4)
    with pytest.raises(ValueError, match="incompatible matmul shapes"):
        L.tape_dryrun(bad_shape.serialize())


@pytest.mark.parametrize("cols", [8, 12, 40, 70, 256, 1000, 8192])
def test_static_bounds_terms_never_skip_a_needed_check(cols):
    """Every bounds test the row compiler emits has the form ((e + 1) * 4NT + off <= lim ||
    var + off < lim); its compile-time left term may replace the runtime test only if every
    slot of step e is in range. Checked by evaluation over all threads t < NT and q < 4 of the
    RMSNorm + SwiGLU gradient tape (row loads, shifted views, reductions, stores) at ragged and
    full widths."""
    import re as _re
    L = _lib()
    tape = J.trace(nn.rms_swiglu_value_and_grad, [(3, cols), (cols,)])
    _, src = L.tape_dryrun(tape.serialize())
    term = _re.compile(r"\(\(e \+ 1\) \* (\d+)LL(?: \+ (-?\d+)LL)? <= (-?\d+)LL \|\| (j|c4 \* 4)(?: \+ (-?\d+)LL)? < (-?\d+)LL\)")
    found = checked = 0
    for kernel in src.split('extern "C"')[1:]:
        nts = set(_re.findall(r"\(\(long long\)e \* (\d+) \+ t\)", kernel)) | set(_re.findall(r"\(long long\)e \* (\d+) \+ t;", kernel))
        assert len(nts) <= 1
        for span, off1, lim1, var, off2, lim2 in term.findall(kernel):
            found += 1
            nt = int(next(iter(nts)))
            span, lim = int(span), int(lim1)
            off = int(off1 or 0)
            assert span == 4 * nt and lim == int(lim2) and off == int(off2 or 0)
            for e in range(lim // span + 2):
                if (e + 1) * span + off > lim:
                    continue
                worst = 4 * (e * nt + nt - 1) + (3 if var == "j" else 0)
                assert worst + off < lim, (cols, span, off, lim, e)
                checked += 1
    # every test was recognised; at widths of whole slot steps the static term decides some
    assert found > 0 and (checked > 0 or cols % 128)
