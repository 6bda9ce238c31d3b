"""Tensor front end: the reference's Tensor API over a chain of SPI backends.

Mirrors core/tensor/Tensor.java:32-557 and the SPI defaults of core/tensor/spi/ComputeBackend.java.
A Tensor is (backend, buffer); every op is one backend call. Transforms (reverse-mode AD),
Vmap (batching) and Jit (fusion + recording) are backends that wrap an inner backend, as the
reference's proxies do, so a tape recorded here has the same calls the reference's
ExecutionPlan records.
"""
from __future__ import annotations

from dataclasses import dataclass

import math
from typing import Sequence

import numpy as np

from . import expr as E


def prod(dims) -> int:
    n = 1
    for d in dims:
        n *= int(d)
    return n


def broadcast_shape(a: tuple, b: tuple) -> tuple:
    """Shape.broadcast (core/tensor/Shape.java:105-121)."""
    rank = max(len(a), len(b))
    out = []
    for i in range(rank):
        da = 1 if i < rank - len(a) else a[i - (rank - len(a))]
        db = 1 if i < rank - len(b) else b[i - (rank - len(b))]
        if da != db and da != 1 and db != 1:
            raise ValueError(f"cannot broadcast shapes {a} and {b}")
        out.append(max(da, db))
    return tuple(out)


def reshape_target(shape: tuple, dims: Sequence[int]) -> tuple:
    """Shape.reshape with one inferred -1 dimension."""
    dims = list(dims)
    total = prod(shape)
    if dims.count(-1) > 1:
        raise ValueError("only one dimension can be inferred")
    if -1 in dims:
        known = prod(d for d in dims if d != -1)
        dims[dims.index(-1)] = total // known if known else 0
    if prod(dims) != total:
        raise ValueError(f"cannot reshape {shape} to {tuple(dims)}")
    return tuple(int(d) for d in dims)


@dataclass(frozen=True)
class ConvSpec:
    """2-D convolution geometry (core/tensor/ConvSpec.java): NCHW images flattened per row."""
    in_channels: int
    in_height: int
    in_width: int
    out_channels: int
    kernel: int
    stride: int = 1
    pad: int = 0

    def __post_init__(self):
        if min(self.in_channels, self.in_height, self.in_width, self.out_channels) < 1:
            raise ValueError("channels and spatial dims must be positive")
        if self.kernel < 1 or self.stride < 1 or self.pad < 0:
            raise ValueError("kernel/stride must be positive, pad non-negative")
        if self.in_height + 2 * self.pad < self.kernel or self.in_width + 2 * self.pad < self.kernel:
            raise ValueError(f"kernel {self.kernel} does not fit {self.in_height}x{self.in_width} with pad {self.pad}")

    @property
    def out_height(self) -> int:
        return (self.in_height + 2 * self.pad - self.kernel) // self.stride + 1

    @property
    def out_width(self) -> int:
        return (self.in_width + 2 * self.pad - self.kernel) // self.stride + 1

    @property
    def input_size(self) -> int:
        return self.in_channels * self.in_height * self.in_width

    @property
    def output_size(self) -> int:
        return self.out_channels * self.out_height * self.out_width

    @property
    def weight_size(self) -> int:
        return self.in_channels * self.kernel * self.kernel

    def weight_shape(self) -> tuple:
        return (self.out_channels, self.weight_size)

    def input_shape(self, batch: int) -> tuple:
        return (batch, self.input_size)

    def output_shape(self, batch: int) -> tuple:
        return (batch, self.output_size)

    def next(self, out_channels: int, kernel: int, stride: int, pad: int) -> "ConvSpec":
        """The spec of a layer that consumes this layer's output."""
        return ConvSpec(self.out_channels, self.out_height, self.out_width, out_channels, kernel, stride, pad)

    def ints(self) -> tuple:
        return (self.in_channels, self.in_height, self.in_width, self.out_channels, self.kernel, self.stride,
                self.pad)

    def batch_of(self, shape: tuple, what: str) -> int:
        if len(shape) != 2:
            raise ValueError(f"{what} must be rank-2, got {shape}")
        return shape[0]


class Buffer:
    """DeviceBuffer (core/tensor/spi/DeviceBuffer.java): anything with a shape."""
    shape: tuple

    @property
    def size(self) -> int:
        return prod(self.shape)


class Backend:
    """The engine SPI with the reference's default implementations where it has them.

    Concrete backends (the oracle's CPU backend, the B200 engine, the tracers) override the
    calls they execute; `fused` defaults to walking the expression with binary/unary/scalar
    calls (ComputeBackend.fused default, ComputeBackend.java:208-237)."""

    def fused(self, expr: E.Expr, inputs: list) -> Buffer:
        memo: dict[int, Buffer] = {}

        def ev(e):
            got = memo.get(id(e))
            if got is not None:
                return got
            if isinstance(e, E.Input):
                r = inputs[e.index]
            elif isinstance(e, E.Unary):
                r = self.unary(e.op, ev(e.a))
            elif isinstance(e, E.Binary):
                r = self.binary(e.op, ev(e.a), ev(e.b))
            else:
                r = self.scalar(e.op, ev(e.a), e.value)
            memo[id(e)] = r
            return r

        return ev(expr)

    def release(self, buf) -> None:
        pass

    def sync(self) -> None:
        pass

    def unwrap(self):
        """The backend this one wraps (tracers), or None for an executing backend."""
        for name in ("inner", "real", "d"):
            b = self.__dict__.get(name)
            if b is not None:
                return b
        return None

    def wraps(self, other) -> bool:
        b = self.unwrap()
        while b is not None:
            if b is other:
                return True
            b = b.unwrap() if isinstance(b, Backend) else None
        return False


def pick_backend(a, b):
    """The backend of a two-operand op: the outer tracer when one operand was captured from
    outside a transform (a constant to it), as a closure over an outer tensor is in JAX."""
    if a is b or not isinstance(b, Backend) or not b.wraps(a):
        return a
    return b


class Tensor:
    """core/tensor/Tensor.java: immutable handle; NumPy broadcasting by explicit broadcastTo."""
    __slots__ = ("backend", "buffer")

    def __init__(self, backend: Backend, buffer: Buffer):
        self.backend = backend
        self.buffer = buffer

    @property
    def shape(self) -> tuple:
        return tuple(self.buffer.shape)

    @property
    def size(self) -> int:
        return prod(self.shape)

    def wrap(self, buf) -> "Tensor":
        return Tensor(self.backend, buf)

    # ---- constants ----
    def full_like(self, value: float) -> "Tensor":
        return self.wrap(self.backend.full(float(value), self.shape))

    # ---- binary with broadcasting (Tensor.java:124-179) ----
    def _binary(self, op: str, other) -> "Tensor":
        if not isinstance(other, Tensor):
            return self.wrap(self.backend.scalar(op, self.buffer, float(other)))
        ls, rs = self.shape, other.shape
        be = pick_backend(self.backend, other.backend)
        if ls == rs:
            return Tensor(be, be.binary(op, self.buffer, other.buffer))
        target = broadcast_shape(ls, rs)
        lb = self.buffer if ls == target else be.broadcast_to(self.buffer, target)
        rb = other.buffer if rs == target else be.broadcast_to(other.buffer, target)
        out = Tensor(be, be.binary(op, lb, rb))
        if lb is not self.buffer:
            be.release(lb)
        if rb is not other.buffer:
            be.release(rb)
        return out

    def add(self, o): return self._binary("ADD", o)
    def sub(self, o): return self._binary("SUB", o)
    def mul(self, o): return self._binary("MUL", o)
    def div(self, o): return self._binary("DIV", o)
    def maximum(self, o): return self._binary("MAX", o)
    def minimum(self, o): return self._binary("MIN", o)

    # ---- unary (Tensor.java:209-247) ----
    def _unary(self, op: str) -> "Tensor":
        return self.wrap(self.backend.unary(op, self.buffer))

    def neg(self): return self._unary("NEG")
    def exp(self): return self._unary("EXP")
    def log(self): return self._unary("LOG")
    def sqrt(self): return self._unary("SQRT")
    def rsqrt(self): return self._unary("RSQRT")
    def tanh(self): return self._unary("TANH")
    def sigmoid(self): return self._unary("SIGMOID")
    def relu(self): return self._unary("RELU")
    def abs(self): return self._unary("ABS")
    def sign(self): return self._unary("SIGN")

    # ---- movement / contraction (Tensor.java:251-398) ----
    def transpose(self) -> "Tensor":
        return self.wrap(self.backend.transpose(self.buffer))

    def matmul(self, o: "Tensor") -> "Tensor":
        be = pick_backend(self.backend, o.backend)
        return Tensor(be, be.matmul(self.buffer, o.buffer))

    def batched_matmul(self, o: "Tensor") -> "Tensor":
        be = pick_backend(self.backend, o.backend)
        return Tensor(be, be.batched_matmul(self.buffer, o.buffer))

    def slice_axis0(self, index: int) -> "Tensor":
        return self.wrap(self.backend.slice_axis0(self.buffer, index))

    def reshape(self, *dims) -> "Tensor":
        if len(dims) == 1 and isinstance(dims[0], (tuple, list)):
            dims = tuple(dims[0])
        return self.wrap(self.backend.reshape(self.buffer, reshape_target(self.shape, dims)))

    def permute(self, *axes) -> "Tensor":
        """Tensor.permute (Tensor.java:346-372): a static reindex gather."""
        if len(axes) == 1 and isinstance(axes[0], (tuple, list)):
            axes = tuple(axes[0])
        rank = len(self.shape)
        if sorted(axes) != list(range(rank)):
            raise ValueError("invalid permutation")
        dims = [self.shape[a] for a in axes]
        # target coordinate j is source axis axes[j]: map = source linear index per target element
        src_strides = [prod(self.shape[d + 1:]) for d in range(rank)]
        idx = np.zeros(dims, dtype=np.int64)
        for j in range(rank):
            shape = [1] * rank
            shape[j] = dims[j]
            idx = idx + src_strides[axes[j]] * np.arange(dims[j], dtype=np.int64).reshape(shape)
        return self.reindex(tuple(dims), idx.reshape(-1))

    def move_axis(self, src: int, dst: int) -> "Tensor":
        """Tensor.moveAxis (Tensor.java:374-389)."""
        rank = len(self.shape)
        src = src + rank if src < 0 else src
        dst = dst + rank if dst < 0 else dst
        axes = [0] * rank
        j = 0
        for i in range(rank):
            if i != dst:
                while j == src:
                    j += 1
                axes[i] = j
                j += 1
        axes[dst] = src
        return self.permute(axes)

    def reindex(self, target, indices) -> "Tensor":
        return self.wrap(self.backend.reindex(self.buffer, tuple(target),
                                              np.asarray(indices, dtype=np.int64)))

    def scatter_add(self, target, indices) -> "Tensor":
        return self.wrap(self.backend.scatter_add(self.buffer, tuple(target),
                                                  np.asarray(indices, dtype=np.int64)))

    # ---- convolution (Tensor.java:400-420) ----
    def conv2d(self, weights: "Tensor", spec: ConvSpec) -> "Tensor":
        be = pick_backend(self.backend, weights.backend)
        return Tensor(be, be.conv2d(self.buffer, weights.buffer, spec))

    def conv2d_grad_input(self, weights: "Tensor", spec: ConvSpec) -> "Tensor":
        """Gradient of conv2d with respect to its input; this is the upstream gradient."""
        be = pick_backend(self.backend, weights.backend)
        return Tensor(be, be.conv2d_grad_input(self.buffer, weights.buffer, spec))

    def conv2d_grad_weight(self, upstream: "Tensor", spec: ConvSpec) -> "Tensor":
        """Gradient of conv2d with respect to its weights; this is the input."""
        be = pick_backend(self.backend, upstream.backend)
        return Tensor(be, be.conv2d_grad_weight(self.buffer, upstream.buffer, spec))

    def relu_backward(self, inp: "Tensor") -> "Tensor":
        be = pick_backend(self.backend, inp.backend)
        return Tensor(be, be.relu_backward(self.buffer, inp.buffer))

    def broadcast_to(self, target) -> "Tensor":
        target = tuple(target)
        return self if self.shape == target else self.wrap(self.backend.broadcast_to(self.buffer, target))

    # ---- reductions (Tensor.java:430-482) ----
    def _axis(self, axis: int) -> int:
        r = len(self.shape)
        n = axis + r if axis < 0 else axis
        if n < 0 or n >= r:
            raise ValueError(f"axis {axis} is out of bounds for shape {self.shape}")
        return n

    def sum(self, axis: int | None = None, keep_dims: bool = False) -> "Tensor":
        if axis is None:
            return self.wrap(self.backend.reduce_sum(self.buffer))
        return self.wrap(self.backend.sum_axis(self.buffer, self._axis(axis), keep_dims))

    def mean(self) -> "Tensor":
        """Tensor.mean (Tensor.java:434-439): sum, then a scalar division by the count."""
        total = self.sum()
        out = total.div(float(self.size))
        self.backend.release(total.buffer)
        return out

    def max(self, axis: int | None = None, keep_dims: bool = False) -> "Tensor":
        if axis is None:
            return self.wrap(self.backend.reduce_max(self.buffer))
        return self.wrap(self.backend.max_axis(self.buffer, self._axis(axis), keep_dims))

    def argmax(self, axis: int) -> "Tensor":
        return self.wrap(self.backend.arg_max_axis(self.buffer, self._axis(axis)))

    def max_axis_backward(self, upstream: "Tensor", axis: int) -> "Tensor":
        be = pick_backend(self.backend, upstream.backend)
        return Tensor(be, be.max_axis_backward(upstream.buffer, self.buffer, self._axis(axis)))

    def close(self) -> None:
        self.backend.release(self.buffer)


def scaled_glorot(fan_in: int, fan_out: int) -> float:
    return math.sqrt(6.0 / (fan_in + fan_out))
