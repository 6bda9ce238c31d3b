"""Deferred execution: whole-plan fusion behind the unmodified SPI.

The reference replays a compiled function one SPI call at a time (ExecutionPlan.execute,
core/tensor/ExecutionPlan.java:96-132, a reflective call per recorded step), and FusingBackend
materialises at every reduction, broadcast and matmul (core/tensor/FusingBackend.java:124-259).
A drop-in backend sees only that call sequence; it cannot change the core. `DeferredBackend`
therefore fuses on its own side of the SPI:

  - every call the engine's tape compiler understands (the tape opcodes of jit.OPCODES) returns a
    lazy buffer and is appended to a pending tape instead of launching;
  - a host read (download), sync, or a call the tape cannot hold (convolutions, quantised
    matrices, random draws) flushes the pending tape: its outputs are the lazy buffers the caller
    still holds (reference counting tells which intermediates are dead), its inputs the concrete
    buffers the calls read;
  - the flushed tape's serialised form (shapes, calls, attributes, data flow) is its signature:
    the first flush of a signature compiles it (j4b_tape_compile: row-fused kernels), every later
    flush with the same signature launches the cached compiled tape with the new inputs.

So a plan replayed call by call, as ExecutionPlan.execute does, runs as the engine's fused row
kernels (the RMSNorm + SwiGLU value-and-gradient tape: one row kernel and one fold) with no
change to the core. Compiled plans are kept in an LRU cache of `max_plans` signatures; a host
scalar that changes every step (a per-step constant recorded into the tape) makes a new
signature, which the cache bounds. Random draws are not deferred: their seeds are attributes of
the tape, and a fresh key each step would compile a new plan each step.
"""
from __future__ import annotations

import weakref
from collections import OrderedDict

from .jit import Call, RecordingBackend, Tape
from .tensor import Buffer


class Lazy(Buffer):
    """A buffer whose value is the output of a pending call; concrete once its tape is flushed."""
    __slots__ = ("shape", "value", "owner", "epoch", "id", "released")

    def __init__(self, shape, owner, epoch, bid):
        self.shape = tuple(int(d) for d in shape)
        self.value = None
        self.owner = owner
        self.epoch = epoch
        self.id = bid
        self.released = False


class DeferredBackend(RecordingBackend):
    """Wraps an executing backend (the engine, or the oracle for CPU checks) behind the same SPI.
    The recording backend's argument checks and shape rules apply to every deferred call, so a
    flushed tape is exactly the tape Jit capture would record for the same calls."""
    executes_tapes = False

    def __init__(self, delegate, max_plans: int = 64, max_pending: int = 4096):
        self.d = delegate
        self.max_plans = max_plans
        self.max_pending = max_pending
        self.plans: OrderedDict = OrderedDict()  # signature -> the delegate's plan dict
        self.stats = {"flushes": 0, "compiled": 0, "replayed": 0, "calls_deferred": 0, "eager_calls": 0}
        self.epoch = 0
        self._reset()

    # ---- the pending tape ----
    def _reset(self):
        self.shapes: list = []
        self.calls: list = []
        self.captured: list = []
        self.inputs: list = []           # (bid, concrete buffer), kept alive until the flush
        self._input_ids: dict = {}       # id(concrete buffer) -> bid
        self.lazies: dict = {}           # bid -> weakref to the Lazy produced by a call
        self.epoch += 1

    def _new_id(self, shape) -> int:
        self.shapes.append(tuple(int(d) for d in shape))
        return len(self.shapes) - 1

    def _concrete(self, b):
        """The executing backend's buffer behind b (flushing if b is still pending)."""
        if isinstance(b, Lazy):
            if b.value is None:
                if b.owner is not self:
                    raise ValueError("lazy buffer of another deferred backend")
                if b.epoch == self.epoch and not b.released:
                    self.flush()
                if b.value is None:
                    raise RuntimeError("a released lazy buffer was read")
            return b.value
        return b

    def _input_id(self, b) -> int:
        if isinstance(b, Lazy) and b.value is None and b.owner is self and b.epoch == self.epoch:
            return b.id
        c = self._concrete(b)
        bid = self._input_ids.get(id(c))
        if bid is None:
            bid = self._new_id(c.shape)
            self._input_ids[id(c)] = bid
            self.inputs.append((bid, c))
        return bid

    def rec(self, call_op: str, shape, ins=(), /, **attrs) -> Lazy:
        """RecordingBackend's hook: every deferred SPI call ends here after its checks."""
        ids = [self._input_id(b) for b in ins]
        bid = self._new_id(shape)
        self.calls.append(Call(call_op, bid, ids, attrs))
        lz = Lazy(shape, self, self.epoch, bid)
        self.lazies[bid] = weakref.ref(lz)
        self.stats["calls_deferred"] += 1
        if len(self.calls) >= self.max_pending:
            self.flush()
        return lz

    def flush(self) -> None:
        """Runs the pending calls as one compiled tape (cached by signature)."""
        if not self.calls:
            return
        live = {}
        for bid, ref in self.lazies.items():
            lz = ref()
            if lz is not None and not lz.released:
                live[bid] = lz
        outs = sorted(live)
        if outs:
            tape = Tape(list(self.shapes), [bid for bid, _ in self.inputs], outs, list(self.calls))
            sig = tape.serialize().tobytes()
            plan = self.plans.get(sig)
            if plan is None:
                plan = {}
                self.plans[sig] = plan
                self.stats["compiled"] += 1
                while len(self.plans) > self.max_plans:
                    self.plans.popitem(last=False)
            else:
                self.plans.move_to_end(sig)
                self.stats["replayed"] += 1
            results = self.d.execute_tape(tape, plan, [c for _, c in self.inputs])
            for bid, r in zip(outs, results):
                live[bid].value = r
        self.stats["flushes"] += 1
        self._reset()

    # ---- SPI: identity, host transfers, lifecycle ----
    def name(self) -> str:
        return self.d.name()

    def upload(self, data, shape=None, *args, **kw):
        return self.d.upload(data, shape, *args, **kw)

    def download(self, b):
        return self.d.download(self._concrete(b))

    def sync(self) -> None:
        self.flush()
        self.d.sync()

    def release(self, b) -> None:
        if isinstance(b, Lazy):
            b.released = True
            if b.value is not None:
                self.d.release(b.value)
                b.value = None
            return
        self.d.release(b)

    def fused_program(self, program, inputs):
        """A `fused` call given as its postfix program (the tape's own encoding)."""
        n = inputs[0].size
        if any(b.size != n for b in inputs):
            raise ValueError("fused inputs must share element count")
        return self.rec("fused", inputs[0].shape, inputs, program=list(program))

    # ---- calls the tape does not hold: flush, then run on the executing backend ----
    def _eager(self, name, *args, **kw):
        self.flush()
        self.stats["eager_calls"] += 1
        args = [self._concrete(a) if isinstance(a, Lazy) else
                [self._concrete(x) if isinstance(x, Lazy) else x for x in a] if isinstance(a, list) else a
                for a in args]
        return getattr(self.d, name)(*args, **kw)

    def random_uniform(self, seed, counter, shape):
        return self._eager("random_uniform", seed, counter, shape)

    def random_normal(self, seed, counter, shape):
        return self._eager("random_normal", seed, counter, shape)

    def conv2d(self, *args, **kw):
        return self._eager("conv2d", *args, **kw)

    def conv2d_grad_input(self, *args, **kw):
        return self._eager("conv2d_grad_input", *args, **kw)

    def conv2d_grad_weight(self, *args, **kw):
        return self._eager("conv2d_grad_weight", *args, **kw)

    # ---- everything else runs on the executing backend, after a flush ----
    def __getattr__(self, name):
        if name.startswith("_") or "d" not in self.__dict__:
            raise AttributeError(name)
        target = getattr(self.d, name)
        if not callable(target):
            return target
        return lambda *args, **kw: self._eager(name, *args, **kw)
