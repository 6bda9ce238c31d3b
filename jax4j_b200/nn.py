"""nn mirrors on the hot path: Dense.forward and FunctionalAdam, plus the two tape workloads.

Dense.forward follows nn/Dense.java:7-14 (reshape -> matmul -> add(bias) -> reshape);
FunctionalAdam follows nn/FunctionalAdam.java:62-107 with the moments and the step counter as
explicit inputs and outputs of one compiled tape.

`mlp_loss` is the 2-layer tanh MLP with softmax cross-entropy that the MLP valueAndGrad + Adam
workload differentiates (the stable softmax of MnistMlp.java:169-187, with a tanh hidden layer
and the loss averaged over the batch). `rms_swiglu_loss` is the vmap-batched RMSNorm + SwiGLU
body: h = x * rsqrt(mean(x^2) + eps) * g per row, split h into halves (a, b), y = silu(a) * b,
loss = mean(y^2).
"""
from __future__ import annotations

import math

from . import jit as J
from . import transforms as T
from . import vmap as V
from .tensor import Tensor


def dense_forward(inp: Tensor, weight: Tensor, bias: Tensor) -> Tensor:
    dims = list(inp.shape)
    if not dims or len(weight.shape) != 2 or dims[-1] != weight.shape[0]:
        raise ValueError("Dense shape mismatch")
    rows = inp.size // dims[-1]
    dims[-1] = weight.shape[1]
    return inp.reshape(rows, weight.shape[0]).matmul(weight).add(bias).reshape(dims)


class FunctionalAdam:
    """Pure Adam: update(params, grads, (m, v, step)) -> (params', (m', v', step'))."""

    def __init__(self, rate: float, beta1: float = .9, beta2: float = .999, epsilon: float = 1e-8):
        if (not (rate > 0) or not math.isfinite(rate) or beta1 < 0 or beta1 >= 1 or beta2 < 0
                or beta2 >= 1 or not (epsilon > 0) or not math.isfinite(epsilon)):
            raise ValueError("invalid Adam hyperparameters")
        self.rate, self.beta1, self.beta2, self.epsilon = rate, beta1, beta2, epsilon
        self.compiled = J.compile(self._step_flat)

    def initialize(self, params: list[Tensor]):
        if not params:
            raise ValueError("Adam requires parameters")
        m = [p.full_like(0) for p in params]
        v = [p.full_like(0) for p in params]
        step = params[0].full_like(0).sum()
        return m, v, step

    def update(self, params, grads, state):
        m, v, step = state
        n = len(params)
        if not (len(grads) == len(m) == len(v) == n):
            raise ValueError("Adam tree structure changed")
        outs = self.compiled(*params, *grads, *m, *v, step)
        return outs[:n], (outs[n:2 * n], outs[2 * n:3 * n], outs[3 * n])

    def _step_flat(self, *flat):
        n = (len(flat) - 1) // 4
        ps, gs, ms, vs, step = flat[:n], flat[n:2 * n], flat[2 * n:3 * n], flat[3 * n:4 * n], flat[-1]
        next_step = step.add(1)
        bc1 = next_step.full_like(1) if self.beta1 == 0 else \
            next_step.mul(math.log(self.beta1)).exp().neg().add(1)
        bc2 = next_step.full_like(1) if self.beta2 == 0 else \
            next_step.mul(math.log(self.beta2)).exp().neg().add(1)
        nm, nv, np_ = [], [], []
        for p, g, m, v in zip(ps, gs, ms, vs):
            if not (p.shape == g.shape == m.shape == v.shape):
                raise ValueError("Adam parameter/gradient/state shapes differ")
            mm = m.mul(self.beta1).add(g.mul(1 - self.beta1))
            vv = v.mul(self.beta2).add(g.mul(g).mul(1 - self.beta2))
            nm.append(mm)
            nv.append(vv)
            np_.append(p.sub(mm.div(bc1).div(vv.div(bc2).sqrt().add(self.epsilon)).mul(self.rate)))
        return [*np_, *nm, *nv, next_step]


def mlp_loss(params: list[Tensor], x: Tensor, onehot: Tensor) -> Tensor:
    w1, b1, w2, b2 = params
    a1 = dense_forward(x, w1, b1).tanh()
    z2 = dense_forward(a1, w2, b2)
    shifted = z2.sub(z2.max(1, True))
    e = shifted.exp()
    probs = e.div(e.sum(1, True))
    return onehot.mul(probs.log()).sum().mul(-1.0 / x.shape[0])


def mlp_value_and_grad(w1, b1, w2, b2, x, onehot):
    """valueAndGrad of mlp_loss over the four parameter leaves: [loss, dW1, db1, dW2, db2]."""
    loss, grads = T.value_and_grad_tree(lambda ps: mlp_loss(ps, x, onehot), [w1, b1, w2, b2])
    return [loss, *grads]


def mlp_train_step(opt: "FunctionalAdam"):
    """One compiled training step of the MLP workload: value and gradient of mlp_loss, then the
    Adam update, as one function of (params, first moments, second moments, step, x, onehot) ->
    [loss, params', m', v', step'] (the shape of the reference's compiled training step,
    TransformsTest.java:455-490)."""

    def step(w1, b1, w2, b2, m1, m2, m3, m4, v1, v2, v3, v4, t, x, onehot):
        loss, grads = T.value_and_grad_tree(lambda ps: mlp_loss(ps, x, onehot), [w1, b1, w2, b2])
        out = opt._step_flat(w1, b1, w2, b2, *grads, m1, m2, m3, m4, v1, v2, v3, v4, t)
        return [loss, *out]

    return step


def rms_swiglu_rows(x: Tensor, g: Tensor, eps: float = 1e-5) -> Tensor:
    """vmap over the rows of x [R, C] of the per-row RMSNorm + SwiGLU body; y [R, C/2]."""
    c = x.shape[1]

    def row(xs):
        xr, gg = xs
        r = xr.mul(xr).mean().add(eps).rsqrt()
        h = xr.mul(r).mul(gg)
        halves = h.reshape(2, c // 2)
        a, b = halves.slice_axis0(0), halves.slice_axis0(1)
        return a.mul(a.sigmoid()).mul(b)

    return V.apply_tree(row, [x, g], [0, None], [0])


def rms_swiglu_loss(x: Tensor, g: Tensor, eps: float = 1e-5) -> Tensor:
    y = rms_swiglu_rows(x, g, eps)
    return y.mul(y).mean()


def rms_swiglu_value_and_grad(x: Tensor, g: Tensor):
    """[loss, dx, dg] of rms_swiglu_loss."""
    loss, (dx, dg) = T.value_and_grad_tree(lambda ps: rms_swiglu_loss(ps[0], ps[1]), [x, g])
    return [loss, dx, dg]


def rms_swiglu_value_and_grad_dp(world: int):
    """Data-parallel shard of the same step: each of `world` ranks holds an equal share of the
    rows; its loss carries the 1/world factor, so summing loss and dg over the ranks gives the
    loss and dg of the whole batch, and each rank's dx is its rows of the whole batch's dx."""
    if world == 1:
        return rms_swiglu_value_and_grad
    inv = 1.0 / world

    def fn(x: Tensor, g: Tensor):
        loss, (dx, dg) = T.value_and_grad_tree(
            lambda ps: rms_swiglu_loss(ps[0], ps[1]).mul(inv), [x, g])
        return [loss, dx, dg]

    return fn
