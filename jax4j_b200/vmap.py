"""Primitive batching as a backend (core/tensor/Vmap.java).

The body runs once; mapped arguments are Batched buffers whose physical buffer carries a
leading batch axis, and each primitive is rewritten onto the physical buffers with the rules of
Vmap.java:176-354 (elementwise ops on broadcast operands, matmul -> batchedMatmul, axis ops at
axis + 1, sliceAxis0 / reindex / scatterAdd with batched index maps, ...). Shared (unmapped)
operands are expanded with reshape + broadcastTo, as Vmap.physical does.
"""
from __future__ import annotations

from typing import Callable

import numpy as np

from .tensor import Backend, Buffer, Tensor, prod


class Batched(Buffer):
    __slots__ = ("owner", "physical", "shape")

    def __init__(self, owner, physical: Buffer, sample_shape: tuple):
        self.owner = owner
        self.physical = physical
        self.shape = tuple(sample_shape)


class BatchingBackend(Backend):
    def __init__(self, real: Backend, batch: int):
        self.real = real
        self.batch = batch

    def _mapped(self, b) -> bool:
        return isinstance(b, Batched) and b.owner is self

    def batch_shape(self, sample) -> tuple:
        return (self.batch,) + tuple(sample)

    def phys(self, b) -> Buffer:
        """Vmap.physical (Vmap.java:150-158)."""
        if self._mapped(b):
            return b.physical
        expanded = self.real.reshape(b, (1,) + tuple(b.shape))
        return self.real.broadcast_to(expanded, self.batch_shape(b.shape))

    def t(self, b) -> Tensor:
        return Tensor(self.real, b)

    # ---- unmapped calls pass through ----
    def full(self, value, shape):
        return self.real.full(value, shape)

    def random_uniform(self, seed, counter, shape):
        return self.real.random_uniform(seed, counter, shape)

    def random_normal(self, seed, counter, shape):
        return self.real.random_normal(seed, counter, shape)

    # ---- elementwise: both operands physical ----
    def binary(self, op, a, b):
        if not (self._mapped(a) or self._mapped(b)):
            return self.real.binary(op, a, b)
        return Batched(self, self.real.binary(op, self.phys(a), self.phys(b)), a.shape)

    def scalar(self, op, a, value):
        if not self._mapped(a):
            return self.real.scalar(op, a, value)
        return Batched(self, self.real.scalar(op, a.physical, value), a.shape)

    def unary(self, op, a):
        if not self._mapped(a):
            return self.real.unary(op, a)
        return Batched(self, self.real.unary(op, a.physical), a.shape)

    def relu_backward(self, up, inp):
        if not (self._mapped(up) or self._mapped(inp)):
            return self.real.relu_backward(up, inp)
        return Batched(self, self.real.relu_backward(self.phys(up), self.phys(inp)), up.shape)

    # ---- shape ops ----
    def reshape(self, a, target):
        if not self._mapped(a):
            return self.real.reshape(a, target)
        return Batched(self, self.real.reshape(a.physical, self.batch_shape(target)), target)

    def broadcast_to(self, a, target):
        if not self._mapped(a):
            return self.real.broadcast_to(a, target)
        target = tuple(target)
        dims = [1] * (len(target) + 1)
        dims[0] = self.batch
        dims[len(dims) - len(a.shape):] = list(a.shape)
        pa = self.real.reshape(a.physical, tuple(dims))
        return Batched(self, self.real.broadcast_to(pa, self.batch_shape(target)), target)

    def transpose(self, a):
        if not self._mapped(a):
            return self.real.transpose(a)
        if len(a.shape) != 2:
            raise ValueError("transpose expects matrix samples")
        r = self.t(a.physical).permute(0, 2, 1)
        return Batched(self, r.buffer, (a.shape[1], a.shape[0]))

    def slice_axis0(self, a, ix):
        if not self._mapped(a):
            return self.real.slice_axis0(a, ix)
        if ix < 0 or ix >= a.shape[0]:
            raise ValueError("slice index")
        sample = a.shape[1:]
        size = prod(sample)
        n = prod(a.shape)
        i = np.arange(self.batch * size, dtype=np.int64)
        idx = (i // size) * n + ix * size + i % size
        return Batched(self, self.real.reindex(a.physical, self.batch_shape(sample), idx), sample)

    # conv2d family: the image batch of a mapped first operand folds into the convolution's own
    # batch when the second operand is shared; otherwise each sample is convolved on its own
    def _conv(self, name, a, b, spec):
        real = self.real
        fn = getattr(real, name)
        if not (self._mapped(a) or self._mapped(b)):
            return fn(a, b, spec)
        if self._mapped(a) and not self._mapped(b) and name != "conv2d_grad_weight":
            n, width = a.shape[0], a.shape[1]
            flat = real.reshape(a.physical, (self.batch * n, width))
            out = fn(flat, b, spec)
            return Batched(self, real.reshape(out, (self.batch, n) + tuple(out.shape[1:])), (n,) + tuple(out.shape[1:]))
        outs = []
        for i in range(self.batch):
            ai = real.slice_axis0(a.physical, i) if self._mapped(a) else a
            bi = real.slice_axis0(b.physical, i) if self._mapped(b) else b
            outs.append(fn(ai, bi, spec))
        return Batched(self, real.stack_axis0(outs), tuple(outs[0].shape))

    def conv2d(self, x, w, spec):
        return self._conv("conv2d", x, w, spec)

    def conv2d_grad_input(self, up, w, spec):
        return self._conv("conv2d_grad_input", up, w, spec)

    def conv2d_grad_weight(self, x, up, spec):
        return self._conv("conv2d_grad_weight", x, up, spec)

    def stack_axis0(self, xs):
        """Stack of samples: the physical [B, ...] buffers stacked to [n, B, ...], gathered to
        [B, n, ...]."""
        if not any(self._mapped(x) for x in xs):
            return self.real.stack_axis0(xs)
        n, bsz = len(xs), self.batch
        sample = tuple(xs[0].shape)
        m = prod(sample)
        st = self.real.stack_axis0([self.phys(x) for x in xs])
        idx = np.arange(bsz * n * m, dtype=np.int64)
        b, rest = np.divmod(idx, n * m)
        j, k = np.divmod(rest, m)
        out = self.real.reindex(st, (bsz, n) + sample, ((j * bsz + b) * m + k).tolist())
        return Batched(self, out, (n,) + sample)

    def _batched_map(self, name, a, target, indices):
        target = tuple(target)
        base = np.asarray(indices, dtype=np.int64)
        m = base.size
        stride = prod(a.shape) if name == "reindex" else prod(target)
        i = np.arange(self.batch * m, dtype=np.int64)
        orig = base[i % m]
        idx = np.where(orig < 0, -1, orig + (i // m) * stride)
        fn = self.real.reindex if name == "reindex" else self.real.scatter_add
        return Batched(self, fn(a.physical, self.batch_shape(target), idx), target)

    def reindex(self, a, target, indices):
        if not self._mapped(a):
            return self.real.reindex(a, target, indices)
        return self._batched_map("reindex", a, target, indices)

    def scatter_add(self, a, target, indices):
        if not self._mapped(a):
            return self.real.scatter_add(a, target, indices)
        return self._batched_map("scatter_add", a, target, indices)

    # ---- contractions ----
    def matmul(self, a, b):
        if not (self._mapped(a) or self._mapped(b)):
            return self.real.matmul(a, b)
        pa, pb = self.phys(a), self.phys(b)
        return Batched(self, self.real.batched_matmul(pa, pb), (a.shape[0], b.shape[1]))

    # ---- reductions ----
    def reduce_sum(self, a):
        if not self._mapped(a):
            return self.real.reduce_sum(a)
        flat = self.real.reshape(a.physical, (self.batch, prod(a.shape)))
        return Batched(self, self.real.sum_axis(flat, 1, True), (1,))

    def reduce_max(self, a):
        if not self._mapped(a):
            return self.real.reduce_max(a)
        flat = self.real.reshape(a.physical, (self.batch, prod(a.shape)))
        return Batched(self, self.real.max_axis(flat, 1, True), (1,))

    @staticmethod
    def _reduced(shape, ax, keep):
        return tuple(1 if i == ax else d for i, d in enumerate(shape)) if keep else \
            tuple(d for i, d in enumerate(shape) if i != ax)

    def sum_axis(self, a, axis, keep):
        if not self._mapped(a):
            return self.real.sum_axis(a, axis, keep)
        return Batched(self, self.real.sum_axis(a.physical, axis + 1, keep),
                       self._reduced(a.shape, axis, keep))

    def sum_axis0(self, a):
        return self.sum_axis(a, 0, False)

    def max_axis(self, a, axis, keep):
        if not self._mapped(a):
            return self.real.max_axis(a, axis, keep)
        return Batched(self, self.real.max_axis(a.physical, axis + 1, keep),
                       self._reduced(a.shape, axis, keep))

    def arg_max_axis(self, a, axis):
        if not self._mapped(a):
            return self.real.arg_max_axis(a, axis)
        return Batched(self, self.real.arg_max_axis(a.physical, axis + 1),
                       self._reduced(a.shape, axis, False))

    def max_axis_backward(self, up, inp, axis):
        if not (self._mapped(up) or self._mapped(inp)):
            return self.real.max_axis_backward(up, inp, axis)
        return Batched(self, self.real.max_axis_backward(self.phys(up), self.phys(inp), axis + 1),
                       inp.shape)

    def download(self, b):
        raise RuntimeError("Host reads inside vmap are unsupported")


def apply_tree(body: Callable[[list], object], inputs: list[Tensor], in_axes: list,
               out_axes: list):
    """Vmap.applyTree (Vmap.java:34-106) over a list of tensors; the body returns a tensor or a
    list of tensors. Null in_axes entries are shared arguments."""
    real = inputs[0].backend
    batch = -1
    for t, ax in zip(inputs, in_axes):
        if ax is not None:
            size = t.shape[ax % len(t.shape)]
            if batch not in (-1, size):
                raise ValueError("mapped axis sizes differ")
            batch = size
    if batch < 0:
        raise ValueError("at least one mapped argument is required")
    vb = BatchingBackend(real, batch)
    wrapped = []
    for t, ax in zip(inputs, in_axes):
        if ax is None:
            wrapped.append(Tensor(vb, t.buffer))
        else:
            ax = ax % len(t.shape)
            phys = t if ax == 0 else t.move_axis(ax, 0)
            wrapped.append(Tensor(vb, Batched(vb, phys.buffer, phys.shape[1:])))
    out = body(wrapped)
    outs = out if isinstance(out, (list, tuple)) else [out]
    if len(outs) != len(out_axes):
        raise ValueError("one out_axis per output leaf required")
    results = []
    for o, ax in zip(outs, out_axes):
        if ax is None:
            if isinstance(o.buffer, Batched) and o.buffer.owner is vb:
                raise ValueError("mapped output requires an out_axis")
            results.append(Tensor(real, o.buffer))
        else:
            t = Tensor(real, vb.phys(o.buffer))
            ax = ax % len(t.shape)
            results.append(t if ax == 0 else t.move_axis(0, ax))
    return results if isinstance(out, (list, tuple)) else results[0]


def apply(body: Callable[[Tensor], Tensor], x: Tensor) -> Tensor:
    """Vmap.apply(body, input) with in/out axis 0."""
    return apply_tree(lambda xs: body(xs[0]), [x], [0], [0])
