"""GPU parity of the scalar-AAD replay engines (`cuda`, `cuda-interp`, `cuda-eager`) against the
CPU oracle (a C restatement of ScalarReplay + Philox, double precision).

Bars, as the reference's CudaScalarReplayTest states them: the random tape's value and gradient
within 2e-5 of the FLOAT64 CPU replay of the same scenarios (both precisions); the closed-form
tape within 2e-4 (FLOAT32) / 1e-10 (FLOAT64). The op-conformance tape: FLOAT32 within
5e-4 + 5e-4 |v| (value) and 5e-3 + 5e-3 |g| (gradients) as AadOpConformanceTest; FLOAT64 within
1e-12 relative -- the same scenarios and the same arithmetic up to libm rounding.
"""
import math

import numpy as np
import pytest
import torch

from jax4j_b200.aad import (AadEngines, AadOptions, AadRecorder, CudaAadEngine, CudaEagerEngine,
                            CudaInterpEngine, Precision)

pytestmark = pytest.mark.gpu

ENGINES = [CudaAadEngine, CudaInterpEngine, CudaEagerEngine]
PRECISIONS = [Precision.FLOAT32, Precision.FLOAT64]


def oracle_means(oracle, tape, paths, offset, seed, inputs=None, threads=8):
    ins = tape.recorded_inputs() if inputs is None else inputs
    v, sq, g = oracle.aad_replay(tape.ops, tape.arg_a, tape.arg_b, tape.constants, ins, tape.input_nodes,
                                 tape.output_nodes, tape.rand_stream_count(), paths, offset, seed, True, threads)
    return v[0] / paths, sq[0] / paths, g[0] / paths


def random_tape():
    def body(rec):
        x = rec.input("x", 2)
        z = rec.randn()
        rec.output(x.mul(z).add(z.mul(z)))
    return AadRecorder.record(body)


def analytic_tape():
    def body(rec):
        x, y = rec.input("x", 2), rec.input("y", 3)
        rec.output(x.mul(x).mul(y).add(x.exp()).add(y.exp()))
    return AadRecorder.record(body)


def conformance_tape():
    """AadOpConformanceTest.everyOp without the uniform draw (these engines decline RANDU)."""
    def body(rec):
        x, y = rec.input("x", 1.3), rec.input("y", 0.7)
        z = rec.randn()
        a = x.add(y).sub(0.1)
        b = x.mul(y).div(x.add(0.5))
        c = a.neg().exp().add(b.abs())
        d = c.add(1.0).log().sqrt()
        e = d.max(z.mul(0.01)).min(x.mul(2.0))
        w = rec.randn()
        rec.output(e.add(w.mul(y)))
    return AadRecorder.record(body)


def asian_tape(steps=64):
    """Arithmetic-average Asian call under geometric Brownian motion (log-Euler steps):
    exp(-r T) max(mean_t S_t - K, 0), inputs S0, K, sigma, r, T."""
    def body(rec):
        s0, k, sig, r, t = (rec.input(n, v) for n, v in
                            (("S0", 100.0), ("K", 100.0), ("sigma", 0.2), ("r", 0.05), ("T", 1.0)))
        dt = t / steps
        drift = (r - sig * sig * 0.5) * dt
        vol = sig * dt.sqrt()
        s, total = s0, rec.constant(0.0)
        for _ in range(steps):
            s = s * (drift + vol * rec.randn()).exp()
            total = total + s
        payoff = (total / steps - k).max(0.0)
        rec.output(payoff * (r.neg() * t).exp())
    return AadRecorder.record(body)


@pytest.mark.parametrize("engine_cls", ENGINES)
@pytest.mark.parametrize("precision", PRECISIONS)
def test_random_replay_matches_cpu(oracle, engine_cls, precision):
    """CudaScalarReplayTest.randomReplayMatchesCpu: 1025 scenarios at offsets 0 and 1031, seed 42."""
    tape = random_tape()
    with engine_cls().compile(tape, AadOptions(precision, True)) as exe:
        assert exe.engine_name() == engine_cls.name
        for offset in (0, 1031):
            v, _, g = oracle_means(oracle, tape, 1025, offset, 42)
            got = exe.replay(1025, offset, 42)
            assert abs(got.value() - v) <= 2e-5, (got.value(), v)
            assert abs(got.gradient("x") - g[0]) <= 2e-5, (got.gradient("x"), g[0])


@pytest.mark.parametrize("engine_cls", ENGINES)
@pytest.mark.parametrize("precision", PRECISIONS)
@pytest.mark.parametrize("adjoints", [True, False])
def test_values_gradients_and_input_updates(engine_cls, precision, adjoints):
    """CudaScalarReplayTest.valuesGradientsAndInputUpdates: closed forms after set_input."""
    tol = 2e-4 if precision == Precision.FLOAT32 else 1e-10
    with engine_cls().compile(analytic_tape(), AadOptions(precision, adjoints)) as exe:
        for x in (2.0, -0.5):
            exe.set_input("x", x)
            r = exe.replay(1025, 17, 42)
            assert abs(r.value() - (x * x * 3 + math.exp(x) + math.exp(3))) <= tol
            if adjoints:
                assert abs(r.gradient("x") - (6 * x + math.exp(x))) <= tol
                assert abs(r.gradient("y") - (x * x + math.exp(3))) <= tol


@pytest.mark.parametrize("engine_cls", ENGINES)
@pytest.mark.parametrize("precision", PRECISIONS)
def test_every_op_matches_the_oracle(oracle, engine_cls, precision):
    tape = conformance_tape()
    n, seed = 200_000, 0x5EED5
    v, _, g = oracle_means(oracle, tape, n, 0, seed)
    with engine_cls().compile(tape, AadOptions(precision, True)) as exe:
        got = exe.replay(n, 0, seed)
    if precision == Precision.FLOAT64:
        # summation order differs (per-thread partials vs one running sum): 1e-12 of the scale
        assert got.value() == pytest.approx(v, rel=1e-12)
        for j, name in enumerate(tape.input_names):
            assert got.gradient(name) == pytest.approx(g[j], rel=1e-12, abs=1e-12)
    else:
        assert abs(got.value() - v) <= 5e-4 + 5e-4 * abs(v)
        for j, name in enumerate(tape.input_names):
            assert abs(got.gradient(name) - g[j]) <= 5e-3 + 5e-3 * abs(g[j])


@pytest.mark.parametrize("engine_cls", ENGINES)
def test_extended_random_and_multi_output_are_declined(engine_cls):
    def uniform(rec):
        rec.output(rec.input("x", 1.0) * rec.randu())

    def streams(rec):
        rec.output(rec.input("x", 1.0) * rec.stream("fx").randn())

    def two(rec):
        x = rec.input("x", 1.0)
        rec.output("a", x * 2.0)
        rec.output("b", x * 3.0)
    for body in (uniform, streams, two):
        with pytest.raises(NotImplementedError, match=engine_cls.name):
            engine_cls().compile(AadRecorder.record(body))


@pytest.mark.parametrize("engine_cls", ENGINES)
def test_replays_are_deterministic_and_report_standard_error(engine_cls):
    with engine_cls().compile(conformance_tape()) as exe:
        a, b = exe.replay(100_003, 11, 7), exe.replay(100_003, 11, 7)
        assert a.value() == b.value() and a.gradients() == b.gradients()
        assert 0 < a.standard_error() < 1e-2


def test_eager_chunks_agree_with_one_pass(oracle):
    """A scratch budget of a few scenarios' worth forces many chunks; FLOAT64 sums agree with
    the single-chunk replay and the oracle."""
    tape = conformance_tape()
    opts = AadOptions(Precision.FLOAT64, True)
    small = opts.with_engine_option("cuda-eager", "bytes", 1000 * tape.size() * 16)
    with CudaEagerEngine().compile(tape, opts) as one, CudaEagerEngine().compile(tape, small) as many:
        assert many.threads_or_slot == 1000 and one.threads_or_slot > 100_000
        a, b = one.replay(33_333, 5, 3), many.replay(33_333, 5, 3)
    v, _, g = oracle_means(oracle, tape, 33_333, 5, 3)
    assert a.value() == pytest.approx(b.value(), rel=1e-13)
    assert a.value() == pytest.approx(v, rel=1e-12)
    np.testing.assert_allclose(a.gradients(), b.gradients(), rtol=1e-13, atol=1e-15)
    np.testing.assert_allclose(a.gradients(), g, rtol=1e-12, atol=1e-12)


def test_interpreter_input_limit():
    def body(rec):
        acc = rec.constant(0.0)
        for i in range(33):
            acc = acc + rec.input(f"x{i}", float(i))
        rec.output(acc)
    with pytest.raises(ValueError, match="at most 32 inputs"):
        CudaInterpEngine().compile(AadRecorder.record(body))
    with CudaAadEngine().compile(AadRecorder.record(body), AadOptions(Precision.FLOAT64)) as exe:
        r = exe.replay(1000, 0, 1)
        assert r.value() == pytest.approx(sum(range(33))) and r.gradients() == [1.0] * 33


@pytest.mark.parametrize("engine_cls", ENGINES)
def test_asian_option_matches_the_oracle(oracle, engine_cls):
    """A 64-step path-dependent tape (~450 nodes, 64 draws): FLOAT64 replay equals the oracle's
    to 1e-12; FLOAT32 within 1e-4 of the value and the gradients' scale."""
    tape = asian_tape()
    n, seed = 20_000, 99
    v, _, g = oracle_means(oracle, tape, n, 1000, seed)
    with engine_cls().compile(tape, AadOptions(Precision.FLOAT64)) as exe:
        r = exe.replay(n, 1000, seed)
        assert r.value() == pytest.approx(v, rel=1e-12)
        np.testing.assert_allclose(r.gradients(), g, rtol=1e-11, atol=1e-13)
    with engine_cls().compile(tape, AadOptions(Precision.FLOAT32)) as exe:
        r = exe.replay(n, 1000, seed)
        assert abs(r.value() - v) <= 1e-4 * abs(v)
        assert np.abs(np.array(r.gradients()) - g).max() <= 1e-4 * np.abs(g).max()


def test_engine_selection_and_replay_safe(oracle, monkeypatch):
    opts = AadOptions(Precision.FLOAT64)
    assert [e.name for e in AadEngines.available(opts)] == ["cuda", "cuda-interp", "cuda-eager"]
    monkeypatch.setenv("NABLATENSOR_ENGINE", "cuda-interp")
    tape = random_tape()
    with AadEngines.compile(tape, opts) as exe:
        assert exe.engine_name() == "cuda-interp"
        exe.set_max_chunk_seconds(0.0005)
        r = exe.replay_safe(300_000, 42)
    v, sq, g = oracle_means(oracle, tape, 300_000, 0, 42)
    assert r.paths == 300_000
    assert r.value() == pytest.approx(v, rel=1e-11) and r.gradient("x") == pytest.approx(g[0], rel=1e-9, abs=1e-14)
    assert r.standard_error() == pytest.approx(math.sqrt((sq - v * v) / 300_000), rel=1e-5)
    monkeypatch.setenv("NABLATENSOR_ENGINE", "cpu")
    with pytest.raises(RuntimeError, match="not usable here"):
        AadEngines.select(opts)


def test_device_launch_is_stream_ordered():
    tape = analytic_tape()
    with CudaAadEngine().compile(tape, AadOptions(Precision.FLOAT64)) as exe:
        ins = torch.tensor([2.0, 3.0], dtype=torch.float64, device="cuda")
        sums = torch.zeros(exe.channels, dtype=torch.float64, device="cuda")
        exe.launch(ins.data_ptr(), 4096, 0, 1, sums.data_ptr(), torch.cuda.current_stream().cuda_stream)
        s = sums.cpu().numpy() / 4096
        assert s[0] == pytest.approx(12 + math.exp(2) + math.exp(3), rel=1e-14)
        assert s[2] == pytest.approx(12 + math.exp(2), rel=1e-14) and s[3] == pytest.approx(4 + math.exp(3), rel=1e-14)


def edge_tape():
    """Repeated operands (x * x, a first contribution that is also accumulated), MAX/MIN between
    active and inactive sides, an unused input, nodes recorded after the output."""
    def body(rec):
        x, y, unused = rec.input("x", 0.3), rec.input("y", 2.0), rec.input("unused", 5.0)
        z = rec.randn()
        w = (x * x + y.exp() * z).max(x * 0.5).min(y) / y + (x - y).abs().sqrt().log()
        rec.output(w)
        w * 3.0 + unused  # after the output: never swept
    return AadRecorder.record(body)


@pytest.mark.parametrize("layout", ["shared", "global"])
def test_interpreter_slot_plan(oracle, layout):
    """The interpreter's liveness-planned slots, in shared memory and in global scratch, against
    the oracle (FLOAT64, 1e-12) on tapes that stress the plan; an unused input's gradient is 0."""
    opts = AadOptions(Precision.FLOAT64)
    if layout == "global":
        opts = opts.with_engine_option("cuda-interp", "threads", 8192)
    for tape in (edge_tape(), conformance_tape(), asian_tape(16)):
        v, _, g = oracle_means(oracle, tape, 50_000, 77, 5)
        with CudaInterpEngine().compile(tape, opts) as exe:
            assert (exe.threads_or_slot == 8192) == (layout == "global")
            r = exe.replay(50_000, 77, 5)
        assert r.value() == pytest.approx(v, rel=1e-12)
        np.testing.assert_allclose(r.gradients(), g, rtol=1e-12, atol=1e-12)
    with CudaInterpEngine().compile(edge_tape(), opts) as exe:
        assert exe.replay(1000, 0, 1).gradient("unused") == 0.0


@pytest.mark.parametrize("engine_cls", ENGINES)
def test_output_is_an_input(engine_cls):
    tape = AadRecorder.record(lambda rec: rec.output(rec.input("x", 1.5)))
    with engine_cls().compile(tape, AadOptions(Precision.FLOAT64)) as exe:
        r = exe.replay(999, 0, 1)
        assert r.value() == 1.5 and r.gradients() == [1.0] and r.standard_error() == 0.0
