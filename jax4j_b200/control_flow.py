"""Structured control flow: cond, while_loop, scan and their tree forms
(core/tensor/ControlFlow.java, DeviceProgram.java).

Predicates are scalar tensors; zero is false. Each region (a branch, a loop test or body, a scan
body) is a function of fixed-shape tensors. Where a region runs depends on the backend of its
operands:

  * an executing backend (the B200 engine): every region is traced once into a tape -- the
    same recording the Jit uses, tensors the region closes over become extra inputs -- and the
    engine compiles it into fused sm_100a kernels (j4b_tape_compile). The loop state stays in
    device memory; the host reads back only the 4-byte predicate of a cond or a while step,
    as the reference's program evaluation does (DeviceProgram.java:334-392). A scan body is
    traced once and launched once per step.
  * reverse-mode differentiation: regions run step by step on the differentiating backend with
    the predicate read from the primal values, so gradients flow through the branch taken and
    through every scan step (higher derivatives nest). A gradient that reaches a while loop
    raises NotImplementedError, as the reference supports only forward-mode derivatives of
    dynamic loops.
  * vmap: a cond with a mapped predicate evaluates both branches batched and selects per sample;
    a while loop runs per sample (each sample keeps its own trip count); a scan runs its body on
    the batched carry.
  * a Jit trace: a cond records both branches and a select on the predicate; a scan's body is
    traced once and its recorded calls are replayed once per step into the enclosing tape; a
    while loop cannot be recorded (its trip count is data), so the compiled function falls back
    to running eagerly for that input signature.
"""
from __future__ import annotations

from typing import Callable, NamedTuple

from . import expr as E
from .tensor import Tensor, prod


class ScanStep(NamedTuple):
    carry: Tensor
    output: Tensor


class ScanResult(NamedTuple):
    carry: Tensor
    outputs: Tensor


class Untraceable(Exception):
    """Raised while recording a region whose control flow depends on data (a while loop)."""


# ---------------------------------------------------------------------------------------------
# backend classification
# ---------------------------------------------------------------------------------------------

def _outer(*ts: Tensor):
    """The backend the operands' ops run on (the outermost transform among them)."""
    from .tensor import pick_backend
    b = ts[0].backend
    for t in ts[1:]:
        b = pick_backend(b, t.backend)
    return b


def _mode(*ts: Tensor) -> str:
    from .jit import FusingBackend, RecordingBackend
    from .transforms import ADBackend
    from .vmap import BatchingBackend
    b = _outer(*ts)
    if isinstance(b, (FusingBackend, RecordingBackend)):
        return "trace"
    if isinstance(b, BatchingBackend):
        return "vmap"
    if isinstance(b, ADBackend):
        return "ad"
    if getattr(b, "executes_tapes", False):
        return "device"
    return "eager"


def _scalar_value(t: Tensor):
    """The predicate's value when it is concrete (through any differentiation layers), else None."""
    from .jit import FusingBackend, RecordingBackend
    from .transforms import ADBackend, Node
    b, buf = t.backend, t.buffer
    while isinstance(b, ADBackend):
        if isinstance(buf, Node) and buf.owner is b:
            buf = buf.primal
        b = b.inner
    if isinstance(b, (FusingBackend, RecordingBackend)):
        return None
    from .vmap import BatchingBackend, Batched
    if isinstance(b, BatchingBackend) and isinstance(buf, Batched) and buf.owner is b:
        return None
    return float(b.download(buf).reshape(-1)[0])


def _select(p: Tensor, yes: Tensor, no: Tensor) -> Tensor:
    """no + [p != 0] (yes - no): the branch chosen by a predicate that is not known here."""
    s = p.abs().sign().reshape(*([1] * len(yes.shape))).broadcast_to(yes.shape)
    return no.add(s.mul(yes.sub(no)))


def _check_scalar(p: Tensor, what: str) -> None:
    if prod(p.shape) != 1:
        raise ValueError(f"{what} predicate must be scalar")


# ---------------------------------------------------------------------------------------------
# regions as compiled tapes (executing backends)
# ---------------------------------------------------------------------------------------------

class _Region:
    """A region traced once into a tape over its explicit input shapes; executed on the
    backend's tape path with the explicit inputs followed by the captured buffers."""

    def __init__(self, fn: Callable, shapes: list):
        from .jit import trace
        self.tape = trace(fn, [tuple(s) for s in shapes])
        self.plan: dict = {}
        self.out_shapes = [tuple(self.tape.shapes[i]) for i in self.tape.outputs]

    def __call__(self, backend, buffers: list) -> list:
        return backend.execute_tape(self.tape, self.plan, list(buffers) + self.tape.captured)


def _regions(backend, *specs):
    """Traces the regions; None when one of them cannot be recorded (then they run eagerly)."""
    try:
        return [_Region(fn, shapes) for fn, shapes in specs]
    except Untraceable:
        return None


# ---------------------------------------------------------------------------------------------
# replay of a recorded tape through a backend (a scan body spliced into an enclosing trace)
# ---------------------------------------------------------------------------------------------

def replay(backend, tape, buffers: list) -> list:
    """Runs the tape's calls on `backend`, one SPI call per recorded call."""
    env = dict(zip(tape.inputs, buffers))
    for c in tape.calls:
        a = [env[i] for i in c.ins]
        shape = tuple(tape.shapes[c.out])
        at = c.attrs
        op = c.op
        if op == "full":
            r = backend.full(at["value"], shape)
        elif op in ("random_uniform", "random_normal"):
            r = getattr(backend, op)(at["seed"], at["counter"], shape)
        elif op == "fused":
            r = backend.fused(E.from_postfix(at["program"]), a)
        elif op == "binary":
            r = backend.binary(at["op"], a[0], a[1])
        elif op == "scalar":
            r = backend.scalar(at["op"], a[0], at["value"])
        elif op == "unary":
            r = backend.unary(at["op"], a[0])
        elif op in ("transpose", "reduce_sum", "reduce_max"):
            r = getattr(backend, op)(a[0])
        elif op in ("matmul", "batched_matmul", "relu_backward"):
            r = getattr(backend, op)(a[0], a[1])
        elif op == "slice_axis0":
            r = backend.slice_axis0(a[0], at["index"])
        elif op == "stack_axis0":
            r = backend.stack_axis0(a)
        elif op in ("sum_axis", "max_axis"):
            r = getattr(backend, op)(a[0], at["axis"], at["keep"])
        elif op == "arg_max_axis":
            r = backend.arg_max_axis(a[0], at["axis"])
        elif op == "max_axis_backward":
            r = backend.max_axis_backward(a[0], a[1], at["axis"])
        elif op in ("reshape", "broadcast_to"):
            r = getattr(backend, op)(a[0], shape)
        elif op in ("reindex", "scatter_add"):
            r = getattr(backend, op)(a[0], shape, at["map"])
        else:
            raise ValueError(f"unknown recorded call {op}")
        env[c.out] = r
    return [env[i] for i in tape.outputs]


# ---------------------------------------------------------------------------------------------
# cond
# ---------------------------------------------------------------------------------------------

def cond(predicate: Tensor, on_true: Callable[[Tensor], Tensor], on_false: Callable[[Tensor], Tensor],
         operand: Tensor) -> Tensor:
    """ControlFlow.cond (ControlFlow.java:15-33): on_true(operand) if predicate != 0 else
    on_false(operand); both branches must produce the same shape."""
    _check_scalar(predicate, "cond")
    mode = _mode(operand, predicate)
    if mode == "device":
        regions = _regions(operand.backend, (on_true, [operand.shape]), (on_false, [operand.shape]))
        if regions is not None:
            yes, no = regions
            if yes.out_shapes[0] != no.out_shapes[0]:
                raise ValueError("cond branch shapes differ")
            taken = yes if operand.backend.download(predicate.buffer).reshape(-1)[0] != 0 else no
            return Tensor(operand.backend, taken(operand.backend, [operand.buffer])[0])
    value = _scalar_value(predicate)
    if value is not None:
        # both branches are checked for shape, as the reference captures both before running one
        chosen = on_true if value != 0 else on_false
        out = chosen(operand)
        other = _shape_of(on_false if value != 0 else on_true, operand)
        if other is not None and tuple(other) != tuple(out.shape):
            raise ValueError("cond branch shapes differ")
        return out
    yes, no = on_true(operand), on_false(operand)
    if tuple(yes.shape) != tuple(no.shape):
        raise ValueError("cond branch shapes differ")
    return _select(predicate, yes, no)


def _shape_of(fn: Callable, operand: Tensor):
    """The output shape of a region without running it on data (a symbolic trace)."""
    from .jit import trace
    try:
        tape = trace(fn, [tuple(operand.shape)])
    except Exception:
        return None
    return tape.shapes[tape.outputs[0]]


# ---------------------------------------------------------------------------------------------
# while
# ---------------------------------------------------------------------------------------------

def while_loop(predicate: Callable[[Tensor], Tensor], body: Callable[[Tensor], Tensor], initial: Tensor) -> Tensor:
    """ControlFlow.whileLoop (ControlFlow.java:35-51): applies body while predicate(carry) != 0;
    the predicate must be scalar and the carry keep its shape."""
    mode = _mode(initial)
    if mode == "trace":
        raise Untraceable("while_loop has a data-dependent trip count")
    if mode == "vmap":
        return _while_mapped(predicate, body, initial)
    if mode == "ad":
        return _while_ad(predicate, body, initial)
    if mode == "device":
        regions = _regions(initial.backend, (predicate, [initial.shape]), (body, [initial.shape]))
        if regions is not None:
            test, step = regions
            if prod(test.out_shapes[0]) != 1:
                raise ValueError("while predicate must be scalar")
            if step.out_shapes[0] != tuple(initial.shape):
                raise ValueError("while carry shape changed")
            be, carry = initial.backend, initial.buffer
            while be.download(test(be, [carry])[0]).reshape(-1)[0] != 0:
                carry = step(be, [carry])[0]
            return Tensor(be, carry)
    return _while_eager(predicate, body, initial)


def _while_eager(predicate, body, carry: Tensor) -> Tensor:
    while True:
        p = predicate(carry)
        _check_scalar(p, "while")
        if _scalar_value(p) == 0:
            return carry
        nxt = body(carry)
        if tuple(nxt.shape) != tuple(carry.shape):
            raise ValueError("while carry shape changed")
        carry = nxt


def _while_ad(predicate, body, initial: Tensor) -> Tensor:
    """Runs the loop on the primal values; the result is a node whose pullback raises."""
    from .transforms import Node
    ad = initial.backend
    buf = initial.buffer
    primal = buf.primal if isinstance(buf, Node) and buf.owner is ad else buf
    out = while_loop(predicate, body, Tensor(ad.inner, primal))

    def pull(_up):
        raise NotImplementedError("Dynamic while loops support forward-mode differentiation only")
    parents = [buf] if isinstance(buf, Node) and buf.owner is ad else []
    return Tensor(ad, Node(ad, out.buffer, parents, pull if parents else None))


def _while_mapped(predicate, body, initial: Tensor) -> Tensor:
    from .vmap import Batched
    bb = initial.backend
    buf = initial.buffer
    if not (isinstance(buf, Batched) and buf.owner is bb):
        return Tensor(bb, while_loop(predicate, body, Tensor(bb.real, buf)).buffer)
    real = Tensor(bb.real, buf.physical)
    outs = [while_loop(predicate, body, Tensor(bb.real, bb.real.slice_axis0(real.buffer, i))).buffer
            for i in range(bb.batch)]
    return Tensor(bb, Batched(bb, bb.real.stack_axis0(outs), initial.shape))


# ---------------------------------------------------------------------------------------------
# scan
# ---------------------------------------------------------------------------------------------

def scan(body: Callable[[Tensor, Tensor], ScanStep], initial: Tensor, xs: Tensor) -> ScanResult:
    """ControlFlow.scan (ControlFlow.java:53-98): carry, y_i = body(carry, xs[i]) for every i
    along axis 0; returns the final carry and the stacked outputs [length, ...]."""
    if len(xs.shape) < 1:
        raise ValueError("scan requires a leading axis")
    length = xs.shape[0]
    sample = tuple(xs.shape[1:])
    mode = _mode(initial, xs)
    if mode in ("device", "trace"):
        def traced(c, x):
            step = body(c, x)
            return [step.carry, step.output]
        try:
            region = _Region(traced, [initial.shape, sample])
        except Untraceable:
            if mode == "trace":
                raise
            region = None
        if region is not None:
            if region.out_shapes[0] != tuple(initial.shape):
                raise ValueError("scan carry shape changed")
            if length == 0:
                raise ValueError("scan requires a non-empty leading axis")
            be = _outer(initial, xs)
            carry, ys = initial.buffer, []
            for i in range(length):
                x = be.slice_axis0(xs.buffer, i)
                carry, y = (region(be, [carry, x]) if mode == "device"
                            else replay(be, region.tape, [carry, x] + region.tape.captured))
                ys.append(y)
            return ScanResult(Tensor(be, carry), Tensor(be, be.stack_axis0(ys)))
    carry, ys = initial, []
    for i in range(length):
        step = body(carry, xs.slice_axis0(i))
        if tuple(step.carry.shape) != tuple(initial.shape):
            raise ValueError("scan carry shape changed")
        carry = step.carry
        ys.append(step.output)
    if not ys:
        raise ValueError("scan requires a non-empty leading axis")
    return ScanResult(carry, _stack(ys))


def _stack(ts: list) -> Tensor:
    b = _outer(*ts)
    return Tensor(b, b.stack_axis0([t.buffer for t in ts]))


# ---------------------------------------------------------------------------------------------
# trees (ControlFlow.condTree / whileTree / scanTree, ControlFlow.java:100-281): the leaves of a
# tree (dicts by sorted key, lists, tuples) are packed into one flat vector, so every region is a
# single-tensor region
# ---------------------------------------------------------------------------------------------

def _flatten(tree):
    """(leaves, rebuild) for a tree of tensors."""
    if isinstance(tree, Tensor):
        return [tree], lambda ls: ls[0]
    if isinstance(tree, dict):
        keys = sorted(tree)
        parts = [_flatten(tree[k]) for k in keys]
        counts = [len(p[0]) for p in parts]

        def rebuild(ls):
            out, i = {}, 0
            for k, (_, rb), n in zip(keys, parts, counts):
                out[k] = rb(ls[i:i + n])
                i += n
            return out
        return [leaf for p in parts for leaf in p[0]], rebuild
    if isinstance(tree, (list, tuple)):
        parts = [_flatten(x) for x in tree]
        counts = [len(p[0]) for p in parts]
        kind = type(tree)

        def rebuild(ls):
            out, i = [], 0
            for (_, rb), n in zip(parts, counts):
                out.append(rb(ls[i:i + n]))
                i += n
            return kind(out) if kind is tuple else out
        return [leaf for p in parts for leaf in p[0]], rebuild
    raise ValueError("control-flow tree requires tensors")


def _spec(tree):
    leaves, rebuild = _flatten(tree)
    return [tuple(t.shape) for t in leaves], rebuild


def pack(tree) -> Tensor:
    """ControlFlow.pack: the leaves' elements, concatenated in flattening order."""
    leaves, _ = _flatten(tree)
    if not leaves:
        raise ValueError("control-flow tree requires tensors")
    total = sum(prod(t.shape) for t in leaves)
    packed, offset = None, 0
    for leaf in leaves:
        n = prod(leaf.shape)
        idx = [-1] * total
        idx[offset:offset + n] = range(n)
        part = leaf.reindex((total,), idx)
        packed = part if packed is None else packed.add(part)
        offset += n
    return packed


def _unpack(packed: Tensor, shapes: list, rebuild):
    leaves, offset = [], 0
    for shp in shapes:
        n = prod(shp)
        leaves.append(packed.reindex(tuple(shp), list(range(offset, offset + n))))
        offset += n
    return rebuild(leaves)


def _unpack_batch(packed: Tensor, shapes: list, rebuild, batch: int):
    total = sum(prod(s) for s in shapes)
    leaves, offset = [], 0
    for shp in shapes:
        n = prod(shp)
        idx = [(i // n) * total + offset + i % n for i in range(batch * n)]
        leaves.append(packed.reindex((batch,) + tuple(shp), idx))
        offset += n
    return rebuild(leaves)


def _check_same(spec, tree):
    if [tuple(t.shape) for t in _flatten(tree)[0]] != spec:
        raise ValueError("control-flow tree structure or shapes changed")


def cond_tree(predicate: Tensor, on_true: Callable, on_false: Callable, operand):
    shapes, rebuild = _spec(operand)
    out_spec = {}

    def packed_branch(fn):
        def run(x):
            value = fn(_unpack(x, shapes, rebuild))
            vs, vr = _spec(value)
            if "shapes" in out_spec and out_spec["shapes"] != vs:
                raise ValueError("control-flow tree structure or shapes changed")
            out_spec.setdefault("shapes", vs)
            out_spec.setdefault("rebuild", vr)
            return pack(value)
        return run
    result = cond(predicate, packed_branch(on_true), packed_branch(on_false), pack(operand))
    return _unpack(result, out_spec["shapes"], out_spec["rebuild"])


def while_tree(predicate: Callable, body: Callable, initial):
    shapes, rebuild = _spec(initial)

    def step(x):
        nxt = body(_unpack(x, shapes, rebuild))
        _check_same(shapes, nxt)
        return pack(nxt)
    result = while_loop(lambda x: predicate(_unpack(x, shapes, rebuild)), step, pack(initial))
    return _unpack(result, shapes, rebuild)


def scan_tree(body: Callable, initial, xs):
    """body(carry_tree, x_tree) -> ScanStep(carry_tree, output_tree); returns
    ScanResult(carry_tree, outputs_tree) with every output leaf stacked along a new axis 0."""
    x_leaves, x_rebuild = _flatten(xs)
    if not x_leaves:
        raise ValueError("scan requires input tensors")
    length = x_leaves[0].shape[0] if x_leaves[0].shape else 0
    samples = []
    for t in x_leaves:
        if len(t.shape) < 1 or t.shape[0] != length:
            raise ValueError("scan axis mismatch")
        samples.append(tuple(t.shape[1:]))
    total = sum(prod(s) for s in samples)
    stacked, offset = None, 0
    for t, smp in zip(x_leaves, samples):
        n = prod(smp)
        idx = [-1] * (length * total)
        for b in range(length):
            idx[b * total + offset:b * total + offset + n] = range(b * n, (b + 1) * n)
        part = t.reindex((length, total), idx)
        stacked = part if stacked is None else stacked.add(part)
        offset += n
    c_shapes, c_rebuild = _spec(initial)
    out_spec = {}

    def packed_body(c, x):
        step = body(_unpack(c, c_shapes, c_rebuild), _unpack(x, samples, x_rebuild))
        _check_same(c_shapes, step.carry)
        os_, orb = _spec(step.output)
        out_spec.setdefault("shapes", os_)
        out_spec.setdefault("rebuild", orb)
        return ScanStep(pack(step.carry), pack(step.output))
    res = scan(packed_body, pack(initial), stacked)
    return ScanResult(_unpack(res.carry, c_shapes, c_rebuild),
                      _unpack_batch(res.outputs, out_spec["shapes"], out_spec["rebuild"], length))
