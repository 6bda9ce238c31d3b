"""Whole-plan fusion behind the unmodified SPI (jax4j_b200/deferred.py).

A recorded plan is replayed one SPI call at a time, as ExecutionPlan.execute does
(ExecutionPlan.java:96-132; oracle/backend.py:replay_tape), on a DeferredBackend:

  CPU  over the oracle backend: results bit-identical to the oracle's own call-by-call replay;
       one flush per host read, one compilation per plan signature, replays hit the cache; dead
       intermediates are not outputs; calls the tape cannot hold flush and run eagerly.
  GPU  over the engine: the RMSNorm + SwiGLU value-and-gradient plan within 1e-4 of the oracle,
       and a cached replay costs exactly the compiled tape's launches (one row kernel + one fold).
"""
import numpy as np
import pytest

from jax4j_b200 import jit as J
from jax4j_b200 import nn
from jax4j_b200.deferred import DeferredBackend, Lazy


def rms_inputs(rows, cols, seed):
    rng = np.random.default_rng(seed)
    return [rng.standard_normal((rows, cols)).astype(np.float32),
            (1 + 0.1 * rng.standard_normal(cols)).astype(np.float32)]


class Spy:
    """Oracle delegate that records every tape it is asked to run."""

    def __init__(self):
        from oracle.backend import OracleBackend
        self.inner = OracleBackend()
        self.tapes = []

    def execute_tape(self, tape, plan, buffers):
        self.tapes.append(tape)
        return self.inner.execute_tape(tape, plan, buffers)

    def __getattr__(self, name):
        return getattr(self.inner, name)


def test_deferred_replay_on_the_oracle(oracle):
    from oracle.backend import replay_tape, run_tape
    tape = J.trace(nn.rms_swiglu_value_and_grad, [(16, 64), (64,)])
    spy = Spy()
    be = DeferredBackend(spy)
    for step, seed in enumerate((1, 2, 3)):
        ins = rms_inputs(16, 64, seed)
        outs = replay_tape(be, tape, [be.upload(a, a.shape) for a in ins])
        assert all(isinstance(o, Lazy) for o in outs) and be.stats["flushes"] == step
        got = [be.download(o) for o in outs]
        for g, w in zip(got, run_tape(tape, ins)):
            assert np.array_equal(g.reshape(-1).view(np.uint32), w.reshape(-1).view(np.uint32))
        assert be.stats["flushes"] == step + 1
    assert be.stats["compiled"] == 1 and be.stats["replayed"] == 2
    assert be.stats["calls_deferred"] == 3 * len(tape.calls)
    # the flushed plan's outputs are exactly the plan's outputs: every intermediate was dead
    assert all(len(t.outputs) == len(tape.outputs) for t in spy.tapes)


def test_deferred_boundaries(oracle):
    from oracle.backend import OracleBackend
    be = DeferredBackend(OracleBackend())
    a = be.upload(np.arange(6, dtype=np.float32), (2, 3))
    b = be.scalar("MUL", a, 2.0)
    c = be.sum_axis(b, 1, False)
    assert isinstance(c, Lazy) and be.stats["flushes"] == 0
    r = be.random_normal(1, 0, (4,))  # not deferred: flushes the pending calls first
    assert be.stats["flushes"] == 1 and be.stats["eager_calls"] == 1 and not isinstance(r, Lazy)
    assert np.array_equal(be.download(c), np.array([6.0, 24.0], np.float32))
    d = be.binary("ADD", c, c)  # a flushed lazy buffer becomes an input of the next tape
    assert np.array_equal(be.download(d), np.array([12.0, 48.0], np.float32))
    e = be.unary("NEG", a)
    be.release(e)
    be.sync()  # nothing live: the pending call is dropped, not run
    with pytest.raises(RuntimeError, match="released"):
        be.download(e)
    with pytest.raises(ValueError, match="shape mismatch"):
        be.binary("ADD", a, be.upload(np.zeros(4, np.float32), (4,)))


@pytest.mark.gpu
def test_deferred_replay_on_the_engine(backend):
    from jax4j_b200 import diagnostics
    from oracle.backend import replay_tape, run_tape
    rows, cols = 256, 1024
    tape = J.trace(nn.rms_swiglu_value_and_grad, [(rows, cols), (cols,)])
    be = DeferredBackend(backend)
    for seed in (5, 6):
        ins = rms_inputs(rows, cols, seed)
        bufs = [be.upload(a, a.shape) for a in ins]
        backend.sync()
        before = diagnostics()["dispatches"]
        outs = replay_tape(be, tape, bufs)
        got = [be.download(o) for o in outs]
        launched = diagnostics()["dispatches"] - before
        for g, w in zip(got, run_tape(tape, ins)):
            g, w = g.reshape(-1).astype(np.float64), w.reshape(-1).astype(np.float64)
            scale = np.abs(w).max()
            assert np.abs(g - w).max() <= 1e-4 * scale + 1e-6
            assert np.linalg.norm(g - w) <= 1e-4 * np.linalg.norm(w)
    handle = next(iter(be.plans.values()))["engine"]
    assert be.stats["compiled"] == 1 and be.stats["replayed"] == 1
    assert handle.stats()["launches"] == 2 and launched == 2  # the cached replay: row kernel + fold
