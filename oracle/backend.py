"""Test infrastructure only: the oracle as an SPI backend, and a tape interpreter.

`OracleBackend` runs every SPI call with the C restatement of CpuBackend (oracle.c), so the
Python front end (Tensor / AD / vmap / Jit tracing) can be checked on the CPU against the
reference's JAX fixtures. `run_tape` interprets a recorded tape call by call with the same
primitives: it is the checker the engine's compiled tapes are compared with. Nothing in the
product imports this module.
"""
from __future__ import annotations

import numpy as np

from jax4j_b200 import expr as E
from jax4j_b200.tensor import Backend, Buffer

from . import oracle as O


class NpBuf(Buffer):
    __slots__ = ("a", "shape")

    def __init__(self, a: np.ndarray):
        self.a = np.ascontiguousarray(a, dtype=np.float32)
        self.shape = tuple(self.a.shape)


def _w(a) -> NpBuf:
    return NpBuf(a)


class OracleBackend(Backend):
    """CpuBackend (CpuBackend.java:61-686) restated over numpy buffers."""
    executes_tapes = True

    def upload(self, host, shape=None) -> NpBuf:
        a = np.asarray(host, dtype=np.float32)
        return _w(a.reshape(shape) if shape is not None else a)

    def download(self, b) -> np.ndarray:
        return b.a.copy()

    def full(self, value, shape):
        return _w(np.full(tuple(shape), np.float32(value), np.float32))

    def random_uniform(self, seed, counter, shape):
        n = int(np.prod(shape, dtype=np.int64))
        return _w(O.random_uniform(seed, counter, n).reshape(shape))

    def random_normal(self, seed, counter, shape):
        n = int(np.prod(shape, dtype=np.int64))
        return _w(O.random_normal(seed, counter, n).reshape(shape))

    def conv2d(self, x, w, spec):
        return _w(O.conv2d(x.a.reshape(x.shape[0], -1), w.a, spec.ints()))

    def conv2d_grad_input(self, up, w, spec):
        return _w(O.conv2d_grad_input(up.a.reshape(up.shape[0], -1), w.a, spec.ints()))

    def conv2d_grad_weight(self, x, up, spec):
        return _w(O.conv2d_grad_weight(x.a.reshape(x.shape[0], -1), up.a.reshape(up.shape[0], -1), spec.ints()))

    def binary(self, op, a, b):
        return _w(O.binary(op, a.a, b.a).reshape(a.shape))

    def scalar(self, op, a, value):
        return _w(O.scalar(op, a.a, value))

    def unary(self, op, a):
        return _w(O.unary(op, a.a))

    def fused(self, expr, inputs):
        n = inputs[0].size
        if any(b.size != n for b in inputs):
            raise ValueError("fused inputs must share element count")
        return _w(O.fused(E.postfix(expr), [b.a.reshape(-1) for b in inputs]).reshape(inputs[0].shape))

    def fused_program(self, program, inputs):
        return _w(O.fused(list(program), [b.a.reshape(-1) for b in inputs]).reshape(inputs[0].shape))

    def transpose(self, a):
        return _w(O.transpose(a.a))

    def matmul(self, a, b):
        return _w(O.matmul(a.a, b.a))

    def batched_matmul(self, a, b):
        return _w(O.batched_matmul(a.a, b.a))

    def slice_axis0(self, a, index):
        if index < 0 or index >= a.shape[0]:
            raise ValueError("index")
        return _w(a.a[index].copy())

    def stack_axis0(self, xs):
        return _w(np.stack([x.a for x in xs]))

    def reduce_sum(self, a):
        return _w(O.reduce_sum(a.a))

    def reduce_max(self, a):
        return _w(O.reduce_max(a.a))

    def sum_axis(self, a, axis, keep):
        return _w(O.sum_axis(a.a, axis, keep))

    def sum_axis0(self, a):
        return self.sum_axis(a, 0, False)

    def max_axis(self, a, axis, keep):
        return _w(O.max_axis(a.a, axis, keep))

    def arg_max_axis(self, a, axis):
        return _w(O.argmax_axis(a.a, axis))

    def max_axis_backward(self, up, inp, axis):
        return _w(O.max_axis_backward(up.a, inp.a, axis))

    def reshape(self, a, target):
        return _w(a.a.reshape(tuple(target)))

    def broadcast_to(self, a, target):
        if a.shape == tuple(target):
            return a
        return _w(O.broadcast_to(a.a, tuple(target)))

    def reindex(self, a, target, indices):
        return _w(O.reindex(a.a, tuple(target), indices))

    def scatter_add(self, a, target, indices):
        return _w(O.scatter_add(a.a, tuple(target), indices))

    def relu_backward(self, up, inp):
        return _w(O.relu_backward(up.a, inp.a))

    def execute_tape(self, tape, plan: dict, buffers: list):
        return [_w(a) for a in run_tape(tape, [b.a for b in buffers])]


def _tensor_map(c):
    return np.asarray(c.attrs["map"], dtype=np.int64)


def replay_tape(be, tape, buffers: list) -> list:
    """ExecutionPlan.execute (ExecutionPlan.java:96-132): the tape's calls replayed one SPI call
    at a time on the backend `be` (any SPI backend with a `fused_program` call); returns the
    output buffers."""
    env: dict = dict(zip(tape.inputs, buffers))
    for c in tape.calls:
        ins = [env[i] for i in c.ins]
        a = c.attrs
        op = c.op
        if op == "full":
            r = be.full(a["value"], tape.shapes[c.out])
        elif op == "fused":
            r = be.fused_program(a["program"], ins)
        elif op in ("random_uniform", "random_normal"):
            r = getattr(be, op)(a["seed"], a["counter"], tape.shapes[c.out])
        elif op in ("binary",):
            r = be.binary(a["op"], *ins)
        elif op == "scalar":
            r = be.scalar(a["op"], ins[0], a["value"])
        elif op == "unary":
            r = be.unary(a["op"], ins[0])
        elif op == "slice_axis0":
            r = be.slice_axis0(ins[0], a["index"])
        elif op == "stack_axis0":
            r = be.stack_axis0(ins)
        elif op in ("sum_axis", "max_axis"):
            r = getattr(be, op)(ins[0], a["axis"], a["keep"])
        elif op == "arg_max_axis":
            r = be.arg_max_axis(ins[0], a["axis"])
        elif op == "max_axis_backward":
            r = be.max_axis_backward(ins[0], ins[1], a["axis"])
        elif op == "reshape":
            r = be.reshape(ins[0], tape.shapes[c.out])
        elif op == "broadcast_to":
            r = be.broadcast_to(ins[0], tape.shapes[c.out])
        elif op in ("reindex", "scatter_add"):
            r = getattr(be, op)(ins[0], tape.shapes[c.out], _tensor_map(c))
        else:
            r = getattr(be, op)(*ins)
        if tuple(r.shape) != tuple(tape.shapes[c.out]):
            raise RuntimeError(f"tape shape mismatch at {op}: {r.shape} vs {tape.shapes[c.out]}")
        env[c.out] = r
    return [env[o] for o in tape.outputs]


def run_tape(tape, inputs: list[np.ndarray]) -> list[np.ndarray]:
    """Interprets a tape (jax4j_b200.jit.Tape) call by call on the oracle: ExecutionPlan.execute
    (ExecutionPlan.java:77-132) with the CPU backend."""
    be = OracleBackend()
    bufs = [_w(np.asarray(x, np.float32).reshape(tape.shapes[bid])) for bid, x in zip(tape.inputs, inputs)]
    return [b.a.copy() for b in replay_tape(be, tape, bufs)]
