"""Reverse-mode autodiff as a backend (core/tensor/Transforms.java).

`value_and_grad` / `grad` / `value_and_grad_tree` run the body once on an AD backend whose
buffers are graph nodes; each primitive computes its local derivative tensors at forward time
and stores a pullback, with the rules of Transforms.java:501-676. `backward` walks the nodes in
reverse topological order (Transforms.java:440-474). All calls land on the inner backend, so under
Jit they are recorded like the reference's calls.
"""
from __future__ import annotations

from typing import Callable

import numpy as np

from .tensor import Backend, Buffer, Tensor, prod


class Node(Buffer):
    __slots__ = ("owner", "primal", "parents", "pull", "shape")

    def __init__(self, owner, primal: Buffer, parents=(), pull=None):
        self.owner = owner
        self.primal = primal
        self.parents = list(parents)
        self.pull = pull
        self.shape = tuple(primal.shape)


def _reduce_to(g: Tensor, target: tuple) -> Tensor:
    """AD.reduceTo (Transforms.java:486-491)."""
    while len(g.shape) > len(target):
        g = g.sum(0)
    for i in range(len(target)):
        if target[i] == 1 and g.shape[i] != 1:
            g = g.sum(i, True)
    return g.reshape(target)


def _last_transpose(t: Tensor) -> Tensor:
    axes = list(range(len(t.shape)))
    axes[-1], axes[-2] = axes[-2], axes[-1]
    return t.permute(axes)


class ADBackend(Backend):
    def __init__(self, inner: Backend):
        self.inner = inner

    def t(self, buf) -> Tensor:
        return Tensor(self.inner, buf)

    def node(self, b) -> Node:
        if isinstance(b, Node) and b.owner is self:
            return b
        return Node(self, b)

    # ---- generic wrapping of one primitive ----
    def _apply(self, name: str, buffers: list, call: Callable[[list], Buffer], rule):
        parents = [self.node(b) for b in buffers]
        out = call([p.primal for p in parents])
        if not parents:
            return Node(self, out)
        a = self.t(parents[0].primal)
        b = self.t(parents[1].primal) if len(parents) > 1 else None
        y = self.t(out)
        pull = rule(a, b, y, parents)
        return Node(self, out, parents, pull)

    # ---- sources (no parents) ----
    def full(self, value, shape):
        return Node(self, self.inner.full(value, shape))

    def random_uniform(self, seed, counter, shape):
        return Node(self, self.inner.random_uniform(seed, counter, shape))

    def random_normal(self, seed, counter, shape):
        return Node(self, self.inner.random_normal(seed, counter, shape))

    # ---- elementwise ----
    def binary(self, op, x, y):
        def rule(a, b, out, parents):
            if op == "ADD":
                da, db = a.full_like(1), b.full_like(1)
            elif op == "SUB":
                da, db = a.full_like(1), b.full_like(-1)
            elif op == "MUL":
                da, db = b, a
            elif op == "DIV":
                da, db = b.full_like(1).div(b), a.neg().div(b.mul(b))
            else:  # MAX, MIN
                sign = a.sub(b).sign().mul(1 if op == "MAX" else -1)
                da, db = sign.add(1).mul(.5), sign.neg().add(1).mul(.5)
            return lambda g: [g.mul(da), g.mul(db)]
        return self._apply("binary", [x, y], lambda p: self.inner.binary(op, p[0], p[1]), rule)

    def scalar(self, op, x, value):
        def rule(a, b, out, parents):
            if op in ("ADD", "SUB"):
                return lambda g: [g]
            if op == "MUL":
                d = a.full_like(float(value))
            elif op == "DIV":
                d = a.full_like(float(1.0 / value))
            else:
                d = a.sub(value).sign().mul(1 if op == "MAX" else -1).add(1).mul(.5)
            return lambda g: [g.mul(d)]
        return self._apply("scalar", [x], lambda p: self.inner.scalar(op, p[0], value), rule)

    def unary(self, op, x):
        def rule(a, b, y, parents):
            d = {
                "NEG": lambda: a.full_like(-1),
                "EXP": lambda: y,
                "LOG": lambda: a.full_like(1).div(a),
                "SQRT": lambda: a.full_like(1).div(y.mul(2)),
                "RSQRT": lambda: y.mul(y).mul(y).mul(-.5),
                "TANH": lambda: y.mul(y).neg().add(1),
                "SIGMOID": lambda: y.mul(y.neg().add(1)),
                "RELU": lambda: a.sign().maximum(0),
                "ABS": lambda: a.sign(),
                "SIGN": lambda: a.full_like(0),
            }[op]()
            return lambda g: [g.mul(d)]
        return self._apply("unary", [x], lambda p: self.inner.unary(op, p[0]), rule)

    # ---- shape ops ----
    def reshape(self, x, target):
        return self._apply("reshape", [x], lambda p: self.inner.reshape(p[0], target),
                           lambda a, b, y, ps: (lambda g: [g.reshape(a.shape)]))

    def reindex(self, x, target, indices):
        return self._apply("reindex", [x], lambda p: self.inner.reindex(p[0], target, indices),
                           lambda a, b, y, ps: (lambda g: [g.scatter_add(a.shape, indices)]))

    def scatter_add(self, x, target, indices):
        return self._apply("scatter_add", [x], lambda p: self.inner.scatter_add(p[0], target, indices),
                           lambda a, b, y, ps: (lambda g: [g.reindex(a.shape, indices)]))

    def transpose(self, x):
        return self._apply("transpose", [x], lambda p: self.inner.transpose(p[0]),
                           lambda a, b, y, ps: (lambda g: [g.transpose()]))

    def broadcast_to(self, x, target):
        return self._apply("broadcast_to", [x], lambda p: self.inner.broadcast_to(p[0], target),
                           lambda a, b, y, ps: (lambda g: [_reduce_to(g, a.shape)]))

    def slice_axis0(self, x, index):
        def rule(a, b, y, ps):
            size = prod(y.shape)
            idx = index * size + np.arange(size, dtype=np.int64)
            return lambda g: [g.scatter_add(a.shape, idx)]
        return self._apply("slice_axis0", [x], lambda p: self.inner.slice_axis0(p[0], index), rule)

    def stack_axis0(self, xs):
        def rule(a, b, y, ps):
            return lambda g: [g.slice_axis0(i) for i in range(len(ps))]
        return self._apply("stack_axis0", list(xs), lambda p: self.inner.stack_axis0(p), rule)

    # ---- reductions ----
    def reduce_sum(self, x):
        return self._apply("reduce_sum", [x], lambda p: self.inner.reduce_sum(p[0]),
                           lambda a, b, y, ps: (lambda g: [g.broadcast_to(a.shape)]))

    def sum_axis(self, x, axis, keep):
        def rule(a, b, y, ps):
            dims = list(a.shape)
            dims[axis] = 1
            return lambda g: [g.reshape(dims).broadcast_to(a.shape)]
        return self._apply("sum_axis", [x], lambda p: self.inner.sum_axis(p[0], axis, keep), rule)

    def sum_axis0(self, x):
        return self.sum_axis(x, 0, False)

    def _max_rule(self, all_: bool, axis: int, keep: bool):
        def rule(a, b, y, ps):
            inp = a.reshape(prod(a.shape)) if all_ else a
            mask = inp.max_axis_backward(y.full_like(1), 0 if all_ else axis).reshape(a.shape)
            dims = list(a.shape)
            if not all_:
                dims[axis] = 1
            if all_:
                return lambda g: [g.broadcast_to(a.shape).mul(mask)]
            return lambda g: [g.reshape(dims).broadcast_to(a.shape).mul(mask)]
        return rule

    def reduce_max(self, x):
        return self._apply("reduce_max", [x], lambda p: self.inner.reduce_max(p[0]),
                           self._max_rule(True, 0, False))

    def max_axis(self, x, axis, keep):
        return self._apply("max_axis", [x], lambda p: self.inner.max_axis(p[0], axis, keep),
                           self._max_rule(False, axis, keep))

    def arg_max_axis(self, x, axis):
        return self._apply("arg_max_axis", [x], lambda p: self.inner.arg_max_axis(p[0], axis),
                           lambda a, b, y, ps: (lambda g: [a.full_like(0)]))

    def max_axis_backward(self, up, inp, axis):
        def rule(a, b, y, ps):
            mask = b.max_axis_backward(a.full_like(1), axis)
            return lambda g: [g.mul(mask).sum(axis).reshape(a.shape), b.full_like(0)]
        return self._apply("max_axis_backward", [up, inp],
                           lambda p: self.inner.max_axis_backward(p[0], p[1], axis), rule)

    def relu_backward(self, up, inp):
        def rule(a, b, y, ps):
            mask = b.sign().maximum(0)
            return lambda g: [g.mul(mask), b.full_like(0)]
        return self._apply("relu_backward", [up, inp],
                           lambda p: self.inner.relu_backward(p[0], p[1]), rule)

    # ---- contractions ----
    # conv2d family (Transforms.java:614-629): each op is bilinear; its two pullbacks are the
    # other two ops of the family
    def conv2d(self, x, w, spec):
        def rule(a, b, out, ps):
            return lambda g: [g.conv2d_grad_input(b, spec), a.conv2d_grad_weight(g, spec)]
        return self._apply("conv2d", [x, w], lambda p: self.inner.conv2d(p[0], p[1], spec), rule)

    def conv2d_grad_input(self, up, w, spec):
        def rule(a, b, out, ps):
            return lambda g: [g.conv2d(b, spec), g.conv2d_grad_weight(a, spec)]
        return self._apply("conv2dGradInput", [up, w], lambda p: self.inner.conv2d_grad_input(p[0], p[1], spec), rule)

    def conv2d_grad_weight(self, x, up, spec):
        def rule(a, b, out, ps):
            return lambda g: [b.conv2d_grad_input(g, spec), a.conv2d(g, spec)]
        return self._apply("conv2dGradWeight", [x, up], lambda p: self.inner.conv2d_grad_weight(p[0], p[1], spec),
                           rule)

    def matmul(self, x, y):
        def rule(a, b, out, ps):
            return lambda g: [_reduce_to(g.matmul(b.transpose()), a.shape),
                              _reduce_to(a.transpose().matmul(g), b.shape)]
        return self._apply("matmul", [x, y], lambda p: self.inner.matmul(p[0], p[1]), rule)

    def batched_matmul(self, x, y):
        def rule(a, b, out, ps):
            return lambda g: [_reduce_to(g.batched_matmul(_last_transpose(b)), a.shape),
                              _reduce_to(_last_transpose(a).batched_matmul(g), b.shape)]
        return self._apply("batched_matmul", [x, y], lambda p: self.inner.batched_matmul(p[0], p[1]), rule)

    def download(self, b):
        raise RuntimeError("Host reads inside differentiation are unsupported")

    # ---- backward pass (Transforms.java:440-474) ----
    def backward(self, ends: list, seeds: list) -> dict:
        topo, seen = [], set()

        def visit(n: Node):
            stack = [(n, False)]
            while stack:
                cur, done = stack.pop()
                if done:
                    topo.append(cur)
                    continue
                if id(cur) in seen:
                    continue
                seen.add(id(cur))
                stack.append((cur, True))
                for p in reversed(cur.parents):
                    if id(p) not in seen:
                        stack.append((p, False))

        for e in ends:
            visit(e)
        grads: dict[int, Tensor] = {}

        def add(node, g):
            cur = grads.get(id(node))
            grads[id(node)] = g if cur is None else cur.add(g)

        for e, s in zip(ends, seeds):
            add(e, s)
        for n in reversed(topo):
            up = grads.get(id(n))
            if up is None or n.pull is None:
                continue
            gs = n.pull(up)
            if len(gs) != len(n.parents):
                raise RuntimeError("pullback arity")
            for p, g in zip(n.parents, gs):
                if g.shape != p.shape:
                    raise ValueError("VJP rule returned an incompatible cotangent")
                add(p, g)
        return grads


def value_and_grad_tree(body: Callable[[list], Tensor], inputs: list[Tensor]):
    """Transforms.valueAndGradTree over a list of tensor leaves: (value, [grads])."""
    inner = inputs[0].backend
    ad = ADBackend(inner)
    leaves = [Node(ad, x.buffer) for x in inputs]
    out = body([Tensor(ad, n) for n in leaves])
    end = ad.node(out.buffer)
    if prod(end.shape) != 1:
        raise ValueError("grad requires scalar output")
    seed = Tensor(inner, end.primal).full_like(1)
    grads = ad.backward([end], [seed])
    gs = []
    for leaf, x in zip(leaves, inputs):
        g = grads.get(id(leaf))
        gs.append(g if g is not None else Tensor(inner, x.buffer).full_like(0))
    return Tensor(inner, end.primal), gs


def value_and_grad(body: Callable[[Tensor], Tensor], x: Tensor):
    """Transforms.valueAndGrad (Transforms.java:30-61)."""
    v, gs = value_and_grad_tree(lambda xs: body(xs[0]), [x])
    return v, gs[0]


def grad(body: Callable[[Tensor], Tensor], x: Tensor) -> Tensor:
    return value_and_grad(body, x)[1]
