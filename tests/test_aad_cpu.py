"""CPU tests of the scalar-AAD engines' host side: the oracle's Philox and replay pinned to
published known answers and closed forms, the recorder and tape bookkeeping, chunk
accumulation, and the generated kernel (validated, emitted and compiled with NVRTC, no GPU)."""
import ctypes
import math

import numpy as np
import pytest

from jax4j_b200 import _lib
from jax4j_b200.aad import (AadOp, AadOptions, AadRecorder, AadResult, Precision, _Accumulator,
                            require_basic_random, require_single_output)


def oracle_result(oracle, tape, paths, offset, seed, inputs=None, threads=1):
    ins = tape.recorded_inputs() if inputs is None else inputs
    v, sq, g = oracle.aad_replay(tape.ops, tape.arg_a, tape.arg_b, tape.constants, ins, tape.input_nodes,
                                 tape.output_nodes, tape.rand_stream_count(), paths, offset, seed, True, threads)
    return v / paths, sq / paths, g / paths


def analytic_tape(x=2.0, y=3.0):
    def body(rec):
        xs, ys = rec.input("x", x), rec.input("y", y)
        rec.output(xs.mul(xs).mul(ys).add(xs.exp()).add(ys.exp()))
    return AadRecorder.record(body)


def random_tape():
    def body(rec):
        x = rec.input("x", 2)
        z = rec.randn()
        rec.output(x.mul(z).add(z.mul(z)))
    return AadRecorder.record(body)


def every_op_tape(with_randu=True):
    """The op-conformance tape of AadOpConformanceTest.everyOp (every AadOp once or more)."""
    def body(rec):
        x, y = rec.input("x", 1.3), rec.input("y", 0.7)
        z = rec.randn()
        a = x.add(y).sub(0.1)
        b = x.mul(y).div(x.add(0.5))
        c = a.neg().exp().add(b.abs())
        d = c.add(1.0).log().sqrt()
        e = d.max(z.mul(0.01)).min(x.mul(2.0))
        if with_randu:
            u = rec.randu()
            rec.output(e.add(u.mul(y)))
        else:
            rec.output(e.add(z.mul(y)))
    return AadRecorder.record(body)


# ---- oracle pins ----

def test_philox_matches_the_published_known_answers(oracle):
    # Random123 philox2x32_10 known-answer vectors (counter, key) -> output
    kat = [((0x00000000, 0x00000000), 0x00000000, (0xff1dae59, 0x6cd10df2)),
           ((0xffffffff, 0xffffffff), 0xffffffff, (0x2c3f628b, 0xab4fd7ad)),
           ((0x243f6a88, 0x85a308d3), 0x13198a2e, (0xdd7ce038, 0xf62a4c12))]
    for (c0, c1), key, want in kat:
        assert oracle.philox2x32_10(c0, c1, key) == want


def draw_tape(k):
    """A tape whose output is draw k of the default stream."""
    def body(rec):
        zs = [rec.randn() for _ in range(k + 1)]
        rec.output(zs[k])
    return AadRecorder.record(body)


def test_replay_draws_are_box_muller_legs_of_philox(oracle):
    """Draw k of scenario p is the cosine (even k) / sine (odd k) leg of Box-Muller on the Philox
    block of counter (lo, hi ^ k // 2) keyed 0x1BD11BDA (Philox.java:36-63)."""
    seed = 0x1234_5678_9ABC_DEF0
    for path in (0, 7, 2 ** 33 + 5):
        lo = (path & 0xFFFFFFFF) ^ (seed & 0xFFFFFFFF)
        hi = (path >> 32) ^ (seed >> 32)
        for k in range(5):
            c0, c1 = oracle.philox2x32_10(lo, hi ^ (k >> 1))
            u1, u2 = (c0 + 0.5) * 2.3283064365386963e-10, (c1 + 0.5) * 2.3283064365386963e-10
            r, ang = math.sqrt(-2.0 * math.log(u1)), 6.283185307179586 * u2
            want = r * (math.sin(ang) if k & 1 else math.cos(ang))
            got, _, _ = oracle_result(oracle, draw_tape(k), 1, path, seed)
            assert got[0] == pytest.approx(want, rel=1e-14, abs=1e-15)


@pytest.mark.parametrize("x", [2.0, -0.5])
def test_oracle_analytic_values_and_gradients(oracle, x):
    """CudaScalarReplayTest.valuesGradientsAndInputUpdates closed forms, FLOAT64 bar 1e-10."""
    tape = analytic_tape()
    v, _, g = oracle_result(oracle, tape, 1025, 17, 42, inputs=[x, 3.0])
    assert abs(v[0] - (x * x * 3 + math.exp(x) + math.exp(3))) <= 1e-10
    assert abs(g[0, 0] - (6 * x + math.exp(x))) <= 1e-10
    assert abs(g[0, 1] - (x * x + math.exp(3))) <= 1e-10


def test_oracle_random_tape_statistics(oracle):
    # E[x z + z^2] = 1 and d/dx = E[z] = 0 for standard normals, within 5 standard errors
    n = 200_000
    v, sq, g = oracle_result(oracle, random_tape(), n, 0, 42, threads=4)
    se = math.sqrt((sq[0] - v[0] ** 2) / n)
    assert abs(v[0] - 1.0) < 5 * se
    assert abs(g[0, 0]) < 5 / math.sqrt(n)


def test_oracle_threads_split_the_range(oracle):
    tape = every_op_tape()
    a = oracle_result(oracle, tape, 3001, 5, 9, threads=1)
    b = oracle_result(oracle, tape, 3001, 5, 9, threads=4)
    for x, y in zip(a, b):
        np.testing.assert_allclose(x, y, rtol=1e-12)


# ---- recorder, tape, options ----

def test_recorder_covers_every_op_and_marks_active_nodes():
    tape = every_op_tape()
    assert {tape.op(i) for i in range(tape.size())} == set(AadOp)
    for i in range(tape.size()):
        op = tape.op(i)
        if op in (AadOp.CONST, AadOp.RANDN, AadOp.RANDU):
            assert not tape.is_active(i)
        if op == AadOp.INPUT:
            assert tape.is_active(i)
    assert tape.input_names == ["x", "y"] and tape.recorded_inputs() == [1.3, 0.7]
    assert tape.has_extended_random() and tape.rand_count() == 1 and tape.rand_total() == 2


def test_constants_streams_outputs_and_errors():
    def body(rec):
        x = rec.input("x", 1.0)
        s = rec.stream("rates")
        rec.output("a", 2.0 * x + s.randn() - 1 / x)
        rec.output("b", abs(-x))
    tape = AadRecorder.record(body)
    assert tape.output_count() == 2 and tape.output_names == ["a", "b"]
    assert tape.rand_stream_count() == 2 and tape.has_extended_random()
    with pytest.raises(NotImplementedError, match="randu\\(\\) or named random streams"):
        require_basic_random(tape, "cuda")
    with pytest.raises(NotImplementedError, match="multi-output"):
        require_single_output(tape, "cuda")
    with pytest.raises(RuntimeError, match="no output"):
        AadRecorder.record(lambda rec: rec.input("x", 1.0))
    with pytest.raises(ValueError, match="recorded twice"):
        AadRecorder.record(lambda rec: [rec.output("v", rec.input("x", 1.0)), rec.output("v", rec.constant(1.0))])
    opts = AadOptions().with_precision(Precision.FLOAT64).with_engine_option("cuda-eager", "bytes", 1 << 20)
    assert opts.precision == Precision.FLOAT64 and opts.engine_options_for("cuda-eager") == {"bytes": str(1 << 20)}
    assert AadOptions.defaults().adjoints and AadOptions.defaults().precision == Precision.FLOAT32


def test_chunk_accumulator_equals_one_replay(oracle):
    """replay_safe's combination of chunk means and standard errors (AadResultAccumulator)
    reproduces the single-replay mean and standard error."""
    tape = random_tape()
    parts, total = [(0, 700), (700, 1300), (2000, 48)], 2048

    def result(offset, count):
        v, sq, g = oracle_result(oracle, tape, count, offset, 3)
        var = (sq[0] * count - count * v[0] ** 2) / (count - 1)
        return AadResult(["value"], [v[0]], [math.sqrt(max(var, 0) / count)], [list(g[0])], ["x"], count, 1.0)

    acc = None
    for off, cnt in parts:
        r = result(off, cnt)
        acc = acc or _Accumulator(r)
        acc.add(r, cnt)
    got, want = acc.result(total), result(0, total)
    assert got.value() == pytest.approx(want.value(), rel=1e-12)
    assert got.standard_error() == pytest.approx(want.standard_error(), rel=1e-9)
    assert got.gradient("x") == pytest.approx(want.gradient("x"), rel=1e-12, abs=1e-15)
    assert got.paths == total and got.seconds == 3.0


# ---- the generated kernel, without a device ----

def dryrun(tape, precision=4, adjoints=1):
    P32 = ctypes.POINTER(ctypes.c_int32)
    arrs = [np.ascontiguousarray(a, np.int32) for a in (tape.ops, tape.arg_a, tape.arg_b)]
    cst = np.ascontiguousarray(tape.constants, np.float64)
    inn = np.ascontiguousarray(tape.input_nodes or [0], np.int32)
    buf = ctypes.create_string_buffer(1 << 20)
    n = ctypes.c_size_t()
    _lib.call("j4b_aad_dryrun", tape.size(), *(a.ctypes.data_as(P32) for a in arrs),
              cst.ctypes.data_as(ctypes.POINTER(ctypes.c_double)), tape.input_count(), inn.ctypes.data_as(P32),
              tape.output_node(), precision, adjoints, buf, len(buf), ctypes.byref(n))
    return buf.value.decode()


@pytest.mark.parametrize("precision", [4, 8])
@pytest.mark.parametrize("adjoints", [0, 1])
def test_generated_kernel_compiles(precision, adjoints):
    src = dryrun(every_op_tape(with_randu=False), precision, adjoints)
    assert ("typedef float real" if precision == 4 else "typedef double real") in src
    assert ("d0 = (real)0" in src) == bool(adjoints)
    # one Philox block serves draws 2m and 2m + 1
    assert src.count("j4b_normal_pair<real>(lo, hi,") == 1


def test_generated_kernel_shares_box_muller_pairs():
    """Each Philox block serves two draws, and pairs of blocks are computed together."""
    def body(rec):
        x = rec.input("x", 1.0)
        acc = x
        for _ in range(7):
            acc = acc * rec.randn()
        rec.output(acc)
    src = dryrun(AadRecorder.record(body))
    # draws 0..6 -> Box-Muller pairs 0..3 -> two interleaved Philox calls covering two pairs each
    assert src.count("j4b_normal_pair2<real>(lo, hi,") == 2 and "j4b_normal_pair<real>(lo" not in src


def test_tape_validation_in_the_abi():
    tape = every_op_tape(with_randu=True)
    with pytest.raises(NotImplementedError, match="randu"):
        dryrun(tape)
    bad = random_tape()
    bad.arg_a = bad.arg_a.copy()
    bad.arg_a[2] = 4  # MUL referring to a later node
    with pytest.raises(ValueError, match="not an earlier node"):
        dryrun(bad)
    with pytest.raises(ValueError, match="precision"):
        dryrun(random_tape(), precision=2)
