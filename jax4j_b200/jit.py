"""Jit: fusion + capture of an SPI call tape, compiled by the engine into fused kernels.

Mirrors core/tensor/Jit.java, FusingBackend.java and ExecutionPlan.java. `compile(fn)` traces
`fn` once per input signature: a FusingBackend folds elementwise ops into Expr chains and
materialises them at fusion boundaries with `fused`, exactly where the reference does; beneath
it a symbolic recording backend (the ExecutionPlan.capture proxy, without executing) appends
every call to a Tape. The engine compiles the tape (j4b_tape_compile) into sm_100a kernels,
fusing row-wise elementwise + reduction groups, and replays it with new inputs
(j4b_tape_launch), the role ExecutionPlan.execute plays in the reference.
"""
from __future__ import annotations

import ctypes
import struct
from dataclasses import dataclass, field
from typing import Callable

import numpy as np

from . import expr as E
from .tensor import Backend, Buffer, Tensor, broadcast_shape, prod

# ---------------------------------------------------------------------------------------------
# the tape
# ---------------------------------------------------------------------------------------------

OPCODES = {
    "full": 1, "fused": 2, "transpose": 3, "matmul": 4, "batched_matmul": 5, "slice_axis0": 6,
    "stack_axis0": 7, "reduce_sum": 8, "reduce_max": 9, "sum_axis": 10, "max_axis": 11,
    "arg_max_axis": 12, "max_axis_backward": 13, "reshape": 14, "broadcast_to": 15,
    "reindex": 16, "scatter_add": 17, "relu_backward": 18, "random_uniform": 19,
    "random_normal": 20, "binary": 21, "scalar": 22, "unary": 23,
}
TAPE_MAGIC = 0x31455041_5442344A  # "J4BTAPE1" little-endian words


class Sym(Buffer):
    """A symbolic buffer of one recorder's tape (shape only)."""
    __slots__ = ("id", "shape", "owner")

    def __init__(self, bid: int, shape: tuple, owner=None):
        self.id = bid
        self.shape = tuple(int(d) for d in shape)
        self.owner = owner


@dataclass
class Call:
    op: str
    out: int
    ins: list
    attrs: dict = field(default_factory=dict)


@dataclass
class Tape:
    shapes: list            # buffer id -> shape
    inputs: list            # buffer ids: the explicit inputs, then one per captured buffer
    outputs: list           # buffer ids
    calls: list             # Call
    captured: list = field(default_factory=list)  # buffers closed over by the traced function

    def serialize(self) -> np.ndarray:
        """int64 words: header, buffer shapes, inputs, outputs, calls (see the engine parser)."""
        w: list[int] = [TAPE_MAGIC, len(self.shapes), len(self.inputs), len(self.outputs),
                        len(self.calls)]
        for s in self.shapes:
            w.append(len(s))
            w.extend(s)
        w.extend(self.inputs)
        w.extend(self.outputs)
        for c in self.calls:
            attrs = encode_attrs(c, self.shapes)
            w.extend((OPCODES[c.op], c.out, len(c.ins)))
            w.extend(c.ins)
            w.append(len(attrs))
            w.extend(attrs)
        return np.asarray(w, dtype=np.int64)


def _f64_bits(v: float) -> int:
    return struct.unpack("<q", struct.pack("<d", float(v)))[0]


def affine_map(target: tuple, m: np.ndarray):
    """(offset, strides) if map[i] = offset + sum_d strides[d] * coord_d(i) over the target
    multi-index, with no -1 entries; else None."""
    m = np.asarray(m, dtype=np.int64)
    if m.size == 0 or (m < 0).any():
        return None
    a = m.reshape(target)
    offset = int(a.reshape(-1)[0])
    strides = []
    for d in range(len(target)):
        if target[d] == 1:
            strides.append(0)
            continue
        idx = [0] * len(target)
        idx[d] = 1
        strides.append(int(a[tuple(idx)]) - offset)
    pred = np.full(target, offset, dtype=np.int64)
    for d, st in enumerate(strides):
        shape = [1] * len(target)
        shape[d] = target[d]
        pred = pred + st * np.arange(target[d], dtype=np.int64).reshape(shape)
    return (offset, strides) if np.array_equal(pred, a) else None


def encode_attrs(c: Call, shapes: list) -> list[int]:
    a = c.attrs
    if c.op == "full":
        return [_f64_bits(a["value"])]
    if c.op == "fused":
        return list(a["program"])
    if c.op == "slice_axis0":
        return [a["index"]]
    if c.op in ("sum_axis", "max_axis"):
        return [a["axis"], int(a["keep"])]
    if c.op in ("arg_max_axis", "max_axis_backward"):
        return [a["axis"]]
    if c.op in ("reindex", "scatter_add"):
        # kind 1: affine over the gather side's multi-index; kind 0: explicit map
        m = np.asarray(a["map"], dtype=np.int64)
        side = shapes[c.out] if c.op == "reindex" else shapes[c.ins[0]]
        aff = affine_map(tuple(side), m)
        if aff is not None:
            off, st = aff
            return [1, off, len(st)] + list(st)
        return [0, int(m.size)] + m.tolist()
    if c.op in ("random_uniform", "random_normal"):
        return [a["seed"], a["counter"]]
    if c.op == "binary" or c.op == "unary":
        return [E.OP[a["op"]]]
    if c.op == "scalar":
        return [E.OP[a["op"]], _f64_bits(a["value"])]
    return []


class RecordingBackend(Backend):
    """ExecutionPlan.capture's recording proxy (ExecutionPlan.java:49-75), symbolic: every call
    returning a buffer is appended to the tape with its inferred shape."""

    def __init__(self):
        self.shapes: list = []
        self.calls: list = []
        self.captured: list = []   # (buffer, Sym) for buffers from outside the traced function
        self._capture_ids: dict = {}

    def new(self, shape) -> Sym:
        s = Sym(len(self.shapes), shape, self)
        self.shapes.append(s.shape)
        return s

    def sym(self, b) -> Sym:
        """This recorder's symbol for b: b itself, or the input that captures a buffer the traced
        function closed over (a constant tensor, or a value of an enclosing trace)."""
        if isinstance(b, Sym) and b.owner is self:
            return b
        got = self._capture_ids.get(id(b))
        if got is None:
            got = self.new(b.shape)
            self._capture_ids[id(b)] = got
            self.captured.append((b, got))
        return got

    def rec(self, call_op: str, shape, ins=(), /, **attrs) -> Sym:
        # positional-only: elementwise calls carry their operator as the attribute `op`
        ids = [self.sym(b).id for b in ins]
        out = self.new(shape)
        self.calls.append(Call(call_op, out.id, ids, attrs))
        return out

    def download(self, b):
        raise RuntimeError("Host reads are not allowed in a compiled JIT function")

    def full(self, value, shape):
        return self.rec("full", shape, value=float(value))

    def random_uniform(self, seed, counter, shape):
        return self.rec("random_uniform", shape, seed=int(seed), counter=int(counter))

    def random_normal(self, seed, counter, shape):
        return self.rec("random_normal", shape, seed=int(seed), counter=int(counter))

    def fused(self, expr, inputs):
        n = inputs[0].size
        if any(b.size != n for b in inputs):
            raise ValueError("fused inputs must share element count")
        return self.rec("fused", inputs[0].shape, inputs, program=E.postfix(expr))

    def binary(self, op, a, b):
        if a.size != b.size:
            raise ValueError(f"shape mismatch: {a.shape} vs {b.shape}")
        return self.rec("binary", a.shape, (a, b), op=op)

    def scalar(self, op, a, value):
        return self.rec("scalar", a.shape, (a,), op=op, value=float(value))

    def unary(self, op, a):
        return self.rec("unary", a.shape, (a,), op=op)

    def transpose(self, a):
        if len(a.shape) != 2:
            raise ValueError(f"transpose requires a rank-2 tensor, got {a.shape}")
        return self.rec("transpose", (a.shape[1], a.shape[0]), (a,))

    def matmul(self, a, b):
        if len(a.shape) != 2 or len(b.shape) != 2 or a.shape[1] != b.shape[0]:
            raise ValueError(f"incompatible matmul shapes: {a.shape} x {b.shape}")
        return self.rec("matmul", (a.shape[0], b.shape[1]), (a, b))

    def batched_matmul(self, a, b):
        if (len(a.shape) != 3 or len(b.shape) != 3 or a.shape[0] != b.shape[0]
                or a.shape[2] != b.shape[1]):
            raise ValueError(f"incompatible batched matmul shapes: {a.shape} x {b.shape}")
        return self.rec("batched_matmul", (a.shape[0], a.shape[1], b.shape[2]), (a, b))

    def slice_axis0(self, a, index):
        if index < 0 or index >= a.shape[0]:
            raise ValueError(f"axis-0 index {index} is out of bounds for {a.shape}")
        return self.rec("slice_axis0", a.shape[1:], (a,), index=int(index))

    def stack_axis0(self, xs):
        return self.rec("stack_axis0", (len(xs),) + xs[0].shape, xs)

    def reduce_sum(self, a):
        return self.rec("reduce_sum", (1,), (a,))

    def reduce_max(self, a):
        return self.rec("reduce_max", (1,), (a,))

    @staticmethod
    def _reduced(shape, axis, keep):
        return tuple(1 if i == axis else d for i, d in enumerate(shape)) if keep else \
            tuple(d for i, d in enumerate(shape) if i != axis)

    def sum_axis(self, a, axis, keep):
        return self.rec("sum_axis", self._reduced(a.shape, axis, keep), (a,), axis=axis, keep=keep)

    def sum_axis0(self, a):
        return self.sum_axis(a, 0, False)

    def max_axis(self, a, axis, keep):
        return self.rec("max_axis", self._reduced(a.shape, axis, keep), (a,), axis=axis, keep=keep)

    def arg_max_axis(self, a, axis):
        return self.rec("arg_max_axis", self._reduced(a.shape, axis, False), (a,), axis=axis)

    def max_axis_backward(self, up, inp, axis):
        return self.rec("max_axis_backward", inp.shape, (up, inp), axis=axis)

    def reshape(self, a, target):
        if prod(target) != a.size:
            raise ValueError(f"cannot reshape {a.shape} to {target}")
        return self.rec("reshape", target, (a,))

    def broadcast_to(self, a, target):
        target = tuple(target)
        if a.shape == target:
            return a
        if broadcast_shape(a.shape, target) != target:
            raise ValueError(f"cannot broadcast shape {a.shape} to {target}")
        return self.rec("broadcast_to", target, (a,))

    def reindex(self, a, target, indices):
        m = np.asarray(indices, dtype=np.int64)
        if m.size != prod(target):
            raise ValueError("index map size")
        if m.size and (m.min() < -1 or m.max() >= a.size):
            raise ValueError("index out of bounds")
        return self.rec("reindex", target, (a,), map=m)

    def scatter_add(self, a, target, indices):
        m = np.asarray(indices, dtype=np.int64)
        if m.size != a.size:
            raise ValueError("index map size")
        if m.size and (m.min() < -1 or m.max() >= prod(target)):
            raise ValueError("index out of bounds")
        return self.rec("scatter_add", target, (a,), map=m)

    def relu_backward(self, up, inp):
        return self.rec("relu_backward", up.shape, (up, inp))

    def _untraceable(self, *args):
        from .control_flow import Untraceable
        raise Untraceable("the tape format has no convolution call")

    conv2d = conv2d_grad_input = conv2d_grad_weight = _untraceable


# ---------------------------------------------------------------------------------------------
# FusingBackend (FusingBackend.java:31-371)
# ---------------------------------------------------------------------------------------------

class ExprBuffer(Buffer):
    __slots__ = ("expr", "leaves", "shape", "materialized", "owner")

    def __init__(self, expr, leaves, shape, owner=None):
        self.expr = expr
        self.leaves = list(leaves)
        self.shape = tuple(shape)
        self.materialized = None  # the delegate's buffer once this chain hit a boundary
        self.owner = owner        # the FusingBackend that built the chain


class FusingBackend(Backend):
    def __init__(self, delegate: Backend):
        self.d = delegate

    def traced(self, b) -> ExprBuffer:
        """b as an expression of this backend; a chain built by another fusing backend (an
        enclosing trace) is a leaf here, materialised by its owner."""
        if isinstance(b, ExprBuffer):
            if b.owner is self or b.owner is None:
                return b
            b = b.owner.materialize(b)
        return ExprBuffer(E.Input(0), [b], b.shape, self)

    def materialize(self, b):
        """FusingBackend.materialize (FusingBackend.java:273-286)."""
        if not isinstance(b, ExprBuffer):
            return b
        if b.owner is not None and b.owner is not self:
            return b.owner.materialize(b)
        if b.materialized is not None:
            return b.materialized
        if isinstance(b.expr, E.Input) and len(b.leaves) == 1:
            return b.leaves[0]
        b.materialized = self.d.fused(b.expr, b.leaves)
        return b.materialized

    @staticmethod
    def merge(left: ExprBuffer, right: ExprBuffer):
        """FusingBackend.merge (FusingBackend.java:318-336): union of leaves by identity."""
        index: dict[int, int] = {}
        leaves: list = []
        for b in left.leaves:
            if id(b) not in index:
                index[id(b)] = len(leaves)
                leaves.append(b)
        mapping = {}
        for i, b in enumerate(right.leaves):
            if id(b) not in index:
                index[id(b)] = len(leaves)
                leaves.append(b)
            mapping[i] = index[id(b)]
        unchanged = all(mapping[i] == i for i in mapping)
        rexpr = right.expr if unchanged else E.remap(right.expr, mapping)
        return left.expr, rexpr, leaves

    # elementwise ops build expressions
    def binary(self, op, a, b):
        la, rb = self.traced(a), self.traced(b)
        le, re_, leaves = self.merge(la, rb)
        return ExprBuffer(E.Binary(op, le, re_), leaves, la.shape, self)

    def scalar(self, op, a, value):
        t = self.traced(a)
        return ExprBuffer(E.Scalar(op, t.expr, float(value)), t.leaves, t.shape, self)

    def unary(self, op, a):
        t = self.traced(a)
        return ExprBuffer(E.Unary(op, t.expr), t.leaves, t.shape, self)

    # everything else is a boundary
    def full(self, value, shape):
        return self.d.full(value, shape)

    def random_uniform(self, seed, counter, shape):
        return self.d.random_uniform(seed, counter, shape)

    def random_normal(self, seed, counter, shape):
        return self.d.random_normal(seed, counter, shape)

    def download(self, b):
        return self.d.download(self.materialize(b))

    def __getattr__(self, name):
        fn = getattr(self.d, name)

        def boundary(*args):
            real = []
            for a in args:
                if isinstance(a, Buffer):
                    real.append(self.materialize(a))
                elif isinstance(a, (list, tuple)) and a and isinstance(a[0], Buffer):
                    real.append([self.materialize(x) for x in a])
                else:
                    real.append(a)
            return fn(*real)

        return boundary


# ---------------------------------------------------------------------------------------------
# capture and compile
# ---------------------------------------------------------------------------------------------

def trace(fn: Callable, input_shapes: list) -> Tape:
    """Runs fn once over symbolic inputs through Fusing + Recording backends (Jit.applyTree,
    Jit.java:125-146) and returns the tape; outputs are materialised as the reference does."""
    rec = RecordingBackend()
    inputs = [rec.new(s) for s in input_shapes]
    fusing = FusingBackend(rec)
    out = fn(*[Tensor(fusing, b) for b in inputs])
    outs = list(out) if isinstance(out, (list, tuple)) else [out]
    out_ids = [rec.sym(fusing.materialize(t.buffer)).id for t in outs]
    return Tape(rec.shapes, [b.id for b in inputs] + [s.id for _, s in rec.captured], out_ids, rec.calls,
                [b for b, _ in rec.captured])


class Compiled:
    """Jit.compile / compileTree (Jit.java:67-114): one engine tape per input signature."""

    def __init__(self, fn: Callable):
        self.fn = fn
        self.plans: dict = {}
        self.traces = 0

    def tape_for(self, shapes: list) -> Tape:
        key = tuple(tuple(s) for s in shapes)
        if self.plans.get(key, {}).get("eager"):
            return None
        if key not in self.plans:
            self.traces += 1
            self.plans[key] = {"tape": trace(self.fn, list(key))}
        return self.plans[key]["tape"]

    def cached_plan_count(self) -> int:
        return len(self.plans)

    def __call__(self, *tensors):
        """Jit.Compiled.apply (Jit.java:80-88): capture on a new signature, then replay. The
        backend executes the tape (`execute_tape`); the plan dict caches what it compiled."""
        backend = tensors[0].backend
        if not getattr(backend, "executes_tapes", False):
            # called while another function is being traced or differentiated: inline
            return self.fn(*tensors)
        shapes = [t.shape for t in tensors]
        key = tuple(tuple(s) for s in shapes)
        from .control_flow import Untraceable
        try:
            tape = self.tape_for(shapes)
        except Untraceable:
            # data-dependent control flow (a while loop): this signature runs eagerly
            self.plans[key] = {"eager": True}
            tape = None
        if tape is None or self.plans[key].get("eager"):
            return self.fn(*tensors)
        outs = backend.execute_tape(tape, self.plans[key], [t.buffer for t in tensors] + tape.captured)
        results = [Tensor(backend, b) for b in outs]
        return results if len(results) > 1 else results[0]


def compile(fn: Callable) -> Compiled:  # noqa: A001 - mirrors Jit.compile
    return Compiled(fn)
