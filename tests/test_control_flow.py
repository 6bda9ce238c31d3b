"""Structured control flow (cond / while_loop / scan and their tree forms) against the known
answers of the reference's TransformsTest (deviceConditionalAndLoop, compiledScanDoesNotUnrollBody,
differentiateDeviceRegions, nestedVmapAndMappedControlFlow, treeControlFlowAndNestedRegions,
higherDerivativesThroughRegionsAndCustomVmap, structuredGradientsAndRuleContracts) and the JAX
fixture scanGradInputs. Each test runs on the oracle backend (CPU) and on the B200 engine, where
regions compile into fused kernels (marked gpu)."""
import numpy as np
import pytest

from jax4j_b200 import control_flow as CF
from jax4j_b200 import jit as J
from jax4j_b200 import transforms as T
from jax4j_b200 import vmap as V
from jax4j_b200.tensor import Tensor


@pytest.fixture(params=["oracle", pytest.param("b200", marks=pytest.mark.gpu)])
def be(request, oracle):
    if request.param == "oracle":
        from oracle.backend import OracleBackend
        return OracleBackend()
    from jax4j_b200.backend import B200Backend
    return B200Backend(0)


def arr(be, x, *shape):
    a = np.asarray(x, np.float32)
    a = a.reshape(shape) if shape else a
    return Tensor(be, be.upload(a, a.shape))


def get(t):
    return np.asarray(t.backend.download(t.buffer)).reshape(-1)


def test_device_conditional_and_loop(be):
    x, p = arr(be, [0], 1), arr(be, [1], 1)
    assert get(CF.cond(p, lambda t: t.add(3), lambda t: t.sub(9), x)).tolist() == [3]
    assert get(CF.cond(arr(be, [0], 1), lambda t: t.add(3), lambda t: t.sub(9), x)).tolist() == [-9]
    loop = CF.while_loop(lambda t: t.neg().add(5).sign().maximum(0), lambda t: t.add(1), x)
    assert get(loop).tolist() == [5]


def test_compiled_scan_does_not_unroll_body(be):
    calls = [0]

    def body(c, x):
        calls[0] += 1
        nxt = c.add(x)
        return CF.ScanStep(nxt, nxt.mul(2))

    plan = J.compile(lambda init, xs: list(CF.scan(body, init, xs)))
    initial, xs = arr(be, [0], 1), arr(be, [1, 2, 3, 4], 4, 1)
    carry, ys = plan(initial, xs)
    assert get(carry).tolist() == [10] and get(ys).tolist() == [2, 6, 12, 20]
    assert calls[0] == 1
    carry, ys = plan(initial, xs)
    assert calls[0] == 1 and plan.traces == 1
    # eager (uncompiled) scan on an executing backend also traces its body once
    calls[0] = 0
    res = CF.scan(body, initial, xs)
    assert get(res.carry).tolist() == [10] and calls[0] == 1


def test_differentiate_device_regions(be):
    initial, xs, p = arr(be, [2], 1), arr(be, [1, 2, 3], 3, 1), arr(be, [1], 1)
    g = T.grad(lambda t: CF.cond(p, lambda x: x.mul(x), lambda x: x.mul(7), t).sum(), initial)
    np.testing.assert_allclose(get(g), [4], atol=1e-5)

    def scan_body(c, x):
        n = c.mul(x)
        return CF.ScanStep(n, n)
    g = T.grad(lambda t: CF.scan(scan_body, t, xs).carry.sum(), initial)
    np.testing.assert_allclose(get(g), [6], atol=1e-5)
    # reverse mode through a dynamic while loop is refused, as in the reference
    with pytest.raises(NotImplementedError, match="forward-mode"):
        T.grad(lambda t: CF.while_loop(lambda x: x.neg().add(10).sign().maximum(0), lambda x: x.mul(2), t).sum(),
               initial)
    # ... but its value is available, and a loop the gradient does not reach is fine
    v = CF.while_loop(lambda x: x.neg().add(10).sign().maximum(0), lambda x: x.mul(2), initial)
    assert get(v).tolist() == [16]
    g = T.grad(lambda t: t.mul(CF.while_loop(lambda x: x.neg().add(10).sign().maximum(0),
                                                 lambda x: x.mul(2), initial)).sum(), initial)
    np.testing.assert_allclose(get(g), [16], atol=1e-5)


def test_scan_gradient_with_respect_to_inputs_matches_jax(be, golden):
    initial, xs = arr(be, [2], 1), arr(be, [1, 2, 3], 3, 1)

    def body(c, v):
        n = c.mul(v)
        return CF.ScanStep(n, n)
    dx = T.grad(lambda t: CF.scan(body, initial, t).carry.sum(), xs)
    np.testing.assert_allclose(get(dx), golden["scanGradInputs"], atol=3e-5, rtol=0)


def test_nested_vmap_and_mapped_control_flow(be):
    x = arr(be, [1, 2, 3, 4, 5, 6, 7, 8], 2, 2, 2)
    loop = V.apply(lambda t: CF.while_loop(lambda v: v.sum().neg().add(9).sign().maximum(0),
                                           lambda v: v.add(1), t), x)
    assert get(loop).tolist() == [1, 2, 3, 4, 5, 6, 7, 8]
    g = T.grad(lambda t: V.apply(lambda v: CF.scan(lambda c, z: CF.ScanStep(c.mul(z), c), v,
                                                   v.reshape(2, 2)).carry, t).sum(), x)
    np.testing.assert_allclose(get(g), [15, 32, 7, 20, 119, 160, 95, 132], atol=1e-5)
    # per-sample trip counts, and a mapped predicate in a cond
    y = arr(be, [1, 7], 2, 1)
    steps = V.apply(lambda t: CF.while_loop(lambda v: v.neg().add(4).sign().maximum(0), lambda v: v.add(1), t), y)
    assert get(steps).tolist() == [4, 7]
    c = V.apply(lambda t: CF.cond(t.add(-1), lambda v: v.mul(10), lambda v: v.sub(1), t), arr(be, [1, 2, 3], 3, 1))
    assert get(c).tolist() == [0, 20, 30]


def test_tree_control_flow_and_nested_regions(be):
    x, y, xs = arr(be, [1], 1), arr(be, [2], 1), arr(be, [1, 2, 3], 3, 1)
    res = CF.while_tree(lambda s: s["a"].neg().add(3).sign().maximum(0),
                        lambda s: {"a": s["a"].add(1), "b": s["b"].mul(2)}, {"a": x, "b": y})
    assert get(res["a"]).tolist() == [3] and get(res["b"]).tolist() == [8]
    nested = CF.while_loop(lambda t: t.neg().add(4).sign().maximum(0),
                           lambda t: CF.cond(t.sign(), lambda v: v.add(1), lambda v: v.add(2), t), x)
    assert get(nested).tolist() == [4]
    sc = CF.scan_tree(lambda c, v: CF.ScanStep({"a": c["a"].add(v["x"]), "b": c["b"].mul(2)}, {"y": c["a"]}),
                      {"a": x, "b": y}, {"x": xs})
    assert get(sc.carry["a"]).tolist() == [7] and get(sc.carry["b"]).tolist() == [16]
    assert get(sc.outputs["y"]).tolist() == [1, 2, 4]
    ct = CF.cond_tree(arr(be, [0], 1), lambda s: {"u": s["u"].mul(2)}, lambda s: {"u": s["u"].add(5)}, {"u": y})
    assert get(ct["u"]).tolist() == [7]


def test_higher_derivatives_through_regions(be):
    x, xs = arr(be, [1, 2], 2), arr(be, [1, 2], 2, 1)

    def step(c, z):
        nxt = c.mul(c).add(z)
        return CF.ScanStep(nxt, nxt)
    second = T.grad(lambda t: T.grad(lambda v: CF.scan(step, v, xs).carry.sum(), t).sum(), x)
    # two steps give (x^2 + 1)^2 + 2; the second derivative is 12 x^2 + 4
    np.testing.assert_allclose(get(second), [16, 52], atol=1e-5)
    cond_second = T.grad(lambda t: T.grad(
        lambda v: CF.cond(v.sum().sign(), lambda a: a.mul(a).mul(a), lambda a: a.mul(a), v).sum(), t).sum(), x)
    np.testing.assert_allclose(get(cond_second), [6, 12], atol=1e-5)


def test_rule_contracts(be):
    x = arr(be, [1, 2], 2)
    with pytest.raises(ValueError, match="carry shape changed"):
        CF.while_loop(lambda t: t.sum(), lambda t: t.sum(), x)
    with pytest.raises(ValueError, match="predicate must be scalar"):
        CF.cond(x, lambda t: t, lambda t: t, x)
    with pytest.raises(ValueError, match="predicate must be scalar"):
        CF.while_loop(lambda t: t, lambda t: t, x)
    with pytest.raises(ValueError, match="branch shapes differ"):
        CF.cond(arr(be, [1], 1), lambda t: t, lambda t: t.sum(), x)
    with pytest.raises(ValueError, match="scan carry shape changed"):
        CF.scan(lambda c, v: CF.ScanStep(c.sum(), c), x, arr(be, [1, 2, 3], 3, 1))


def test_jit_with_while_runs_eagerly_and_closures_are_captured(be):
    w = arr(be, [10, 20], 2)
    plan = J.compile(lambda t: CF.while_loop(lambda v: v.sum().neg().add(50).sign().maximum(0),
                                             lambda v: v.add(w), t))
    out = plan(arr(be, [1, 1], 2))
    assert get(out).tolist() == [21, 41]
    closure = J.compile(lambda t: t.mul(w).add(1))
    assert get(closure(arr(be, [1, 2], 2))).tolist() == [11, 41]
    assert get(closure(arr(be, [3, 3], 2))).tolist() == [31, 61]


def test_packed_tree_regions_compile_for_the_engine(oracle):
    """The tree forms' pack / unpack regions (reindex views with padding over width-1 values)
    plan and compile with the engine's tape compiler (j4b_tape_dryrun: NVRTC, no device)."""
    import ctypes
    from jax4j_b200 import _lib
    from oracle.backend import OracleBackend
    be = OracleBackend()
    tapes = []
    init = CF._Region.__init__

    def spy(self, fn, shapes):
        init(self, fn, shapes)
        tapes.append(self.tape)
    CF._Region.__init__ = spy
    try:
        x, y, xs = arr(be, [1], 1), arr(be, [2], 1), arr(be, [1, 2, 3], 3, 1)
        CF.while_tree(lambda s: s["a"].neg().add(3).sign().maximum(0),
                      lambda s: {"a": s["a"].add(1), "b": s["b"].mul(2)}, {"a": x, "b": y})
        CF.scan_tree(lambda c, v: CF.ScanStep({"a": c["a"].add(v["x"]), "b": c["b"].mul(2)}, {"y": c["a"]}),
                     {"a": x, "b": y}, {"x": xs})
    finally:
        CF._Region.__init__ = init
    assert len(tapes) == 3
    for t in tapes:
        w = t.serialize()
        st = _lib.TapeStats()
        n = ctypes.c_size_t()
        _lib.call("j4b_tape_dryrun", w.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)), w.size, ctypes.byref(st),
                  None, 0, ctypes.byref(n))
        assert st.groups >= 1
