"""Scalar-AAD Monte-Carlo replay on the B200: record a scalar computation once, replay it for
millions of random scenarios with adjoint (reverse-mode) gradients, on one of three engines.

Mirrors the reference's engine package (core/engine/):
  * AadRecorder / SDouble (AadRecorder.java, SDouble.java): record inputs, constants,
    standard-normal draws and the ops of AadOp.java into an AadTape;
  * AadTape (AadTape.java): the node arrays, active flags, random-stream bookkeeping;
  * AadOptions (AadOptions.java): working precision, adjoints on/off, per-engine options;
  * AadEngine implementations `cuda` (per-tape generated kernel), `cuda-interp` (fixed
    interpreter kernel) and `cuda-eager` (one launch per node), priorities 100 / 90 / 80 as
    CudaAadEngine.java, CudaInterpEngine.java, CudaEagerEngine.java;
  * AadEngines (AadEngines.java): discovery, selection (environment variable
    NABLATENSOR_ENGINE in place of -Dnablatensor.engine), compile;
  * AadExecutable (AadExecutable.java, AbstractAadExecutable.java): set_input, replay, and the
    chunked replay_safe / calibrate built on the measured rate;
  * AadResult (AadResult.java) and the chunk accumulator (AadResultAccumulator.java).

The engines run in libjax4j_b200.so (csrc/aad.cu); there is no CPU engine here (the CPU
replay the results are checked against lives in the test oracle). Unlike the reference's CUDA
engines, these also sum the squared output, so a replay reports its standard error.
"""
from __future__ import annotations

import ctypes
import enum
import math
import os
import time
from dataclasses import dataclass, field, replace

import numpy as np

from ._lib import call, load


class AadOp(enum.IntEnum):
    """Node kinds; the ordinals are the op codes of the C ABI (AadOp.java:22-37)."""
    CONST = 0
    INPUT = 1
    RANDN = 2
    RANDU = 3
    ADD = 4
    SUB = 5
    MUL = 6
    DIV = 7
    NEG = 8
    EXP = 9
    LOG = 10
    SQRT = 11
    MAX = 12
    MIN = 13
    ABS = 14


_UNARY = {AadOp.NEG, AadOp.EXP, AadOp.LOG, AadOp.SQRT, AadOp.ABS}


class Precision(enum.Enum):
    FLOAT32 = 4
    FLOAT64 = 8


@dataclass(frozen=True)
class AadOptions:
    """Replay settings (AadOptions.java:37-113). `threads` is kept for CPU engines and ignored
    here; `engine_options` maps an engine name to its own {key: value} options: `cuda-interp`
    reads "threads" (scratch rows), `cuda-eager` reads "bytes" (scratch budget per chunk)."""
    precision: Precision = Precision.FLOAT32
    adjoints: bool = True
    threads: int = 0
    engine_options: dict = field(default_factory=dict)

    @staticmethod
    def defaults() -> "AadOptions":
        return AadOptions()

    def with_precision(self, value: Precision) -> "AadOptions":
        return replace(self, precision=value)

    def with_adjoints(self, value: bool) -> "AadOptions":
        return replace(self, adjoints=value)

    def with_threads(self, value: int) -> "AadOptions":
        return replace(self, threads=value)

    def with_engine_option(self, engine: str, key: str, value: str) -> "AadOptions":
        opts = {e: dict(m) for e, m in self.engine_options.items()}
        opts.setdefault(engine, {})[key] = str(value)
        return replace(self, engine_options=opts)

    def engine_options_for(self, engine: str) -> dict:
        return dict(self.engine_options.get(engine, {}))

    def resolved_threads(self) -> int:
        return self.threads if self.threads > 0 else (os.cpu_count() or 1)


# ---------------------------------------------------------------------------------------------
# recording
# ---------------------------------------------------------------------------------------------

class SDouble:
    """A recorded scalar (SDouble.java): every operation appends a node to the recorder's tape.
    Plain numbers on either side become CONST nodes."""
    __slots__ = ("rec", "node")

    def __init__(self, rec: "AadRecorder", node: int):
        self.rec, self.node = rec, node

    def _lift(self, other) -> "SDouble":
        if isinstance(other, SDouble):
            if other.rec is not self.rec:
                raise ValueError("operands come from different recordings")
            return other
        return self.rec.constant(float(other))

    def _bin(self, op: AadOp, other) -> "SDouble":
        return self.rec._node(op, self.node, self._lift(other).node)

    def add(self, other): return self._bin(AadOp.ADD, other)
    def sub(self, other): return self._bin(AadOp.SUB, other)
    def mul(self, other): return self._bin(AadOp.MUL, other)
    def div(self, other): return self._bin(AadOp.DIV, other)
    def max(self, other): return self._bin(AadOp.MAX, other)
    def min(self, other): return self._bin(AadOp.MIN, other)
    def neg(self): return self.rec._node(AadOp.NEG, self.node, -1)
    def exp(self): return self.rec._node(AadOp.EXP, self.node, -1)
    def log(self): return self.rec._node(AadOp.LOG, self.node, -1)
    def sqrt(self): return self.rec._node(AadOp.SQRT, self.node, -1)
    def abs(self): return self.rec._node(AadOp.ABS, self.node, -1)

    __add__ = add
    __sub__ = sub
    __mul__ = mul
    __truediv__ = div
    __neg__ = neg
    __abs__ = abs

    def __radd__(self, other): return self._lift(other).add(self)
    def __rsub__(self, other): return self._lift(other).sub(self)
    def __rmul__(self, other): return self._lift(other).mul(self)
    def __rtruediv__(self, other): return self._lift(other).div(self)


class AadRecorder:
    """Records one scalar computation (AadRecorder.java): `AadRecorder.record(body)` calls
    body(rec) and returns the tape."""

    def __init__(self):
        self._op, self._a, self._b, self._cst = [], [], [], []
        self._in_nodes, self._in_names, self._in_values = [], [], []
        self._streams = ["default"]
        self._counts = [[0, 0]]  # [normal, uniform] per stream
        self._out_nodes, self._out_names = [], []

    @staticmethod
    def record(body) -> "AadTape":
        rec = AadRecorder()
        body(rec)
        return rec._build()

    def _add(self, op: AadOp, a: int, b: int, value: float = 0.0) -> int:
        self._op.append(int(op))
        self._a.append(a)
        self._b.append(b)
        self._cst.append(value)
        return len(self._op) - 1

    def _node(self, op: AadOp, a: int, b: int) -> SDouble:
        return SDouble(self, self._add(op, a, b))

    def input(self, name: str, value: float) -> SDouble:
        node = self._add(AadOp.INPUT, len(self._in_nodes), -1, float(value))
        self._in_nodes.append(node)
        self._in_names.append(name)
        self._in_values.append(float(value))
        return SDouble(self, node)

    def constant(self, value: float) -> SDouble:
        return SDouble(self, self._add(AadOp.CONST, -1, -1, float(value)))

    def _stream(self, name: str) -> int:
        if name in self._streams:
            return self._streams.index(name)
        self._streams.append(name)
        self._counts.append([0, 0])
        return len(self._streams) - 1

    def _draw(self, kind: int, stream: str) -> SDouble:
        si = self._stream(stream)
        ordinal = self._counts[si][kind]
        self._counts[si][kind] += 1
        return SDouble(self, self._add(AadOp.RANDN if kind == 0 else AadOp.RANDU, ordinal, si))

    def randn(self) -> SDouble:
        return self._draw(0, "default")

    def randu(self) -> SDouble:
        return self._draw(1, "default")

    def stream(self, name: str) -> "RandomStream":
        if not name or not name.strip():
            raise ValueError("stream name must be non-blank")
        return RandomStream(self, name)

    def output(self, name_or_value, value: SDouble | None = None) -> None:
        name, v = ("value", name_or_value) if value is None else (name_or_value, value)
        if name in self._out_names:
            raise ValueError(f"output '{name}' recorded twice")
        self._out_names.append(name)
        self._out_nodes.append(v.node)

    def _build(self) -> "AadTape":
        if not self._out_nodes:
            raise RuntimeError("no output was recorded")
        return AadTape(np.array(self._op, np.int32), np.array(self._a, np.int32), np.array(self._b, np.int32),
                       np.array(self._cst, np.float64), list(self._in_nodes), list(self._in_names),
                       list(self._in_values), list(self._streams), [c[0] for c in self._counts],
                       [c[1] for c in self._counts], list(self._out_nodes), list(self._out_names))


class RandomStream:
    """A named, independent random stream (AadRecorder.RandomStream)."""

    def __init__(self, rec: AadRecorder, name: str):
        self.rec, self.name = rec, name

    def randn(self) -> SDouble:
        return self.rec._draw(0, self.name)

    def randu(self) -> SDouble:
        return self.rec._draw(1, self.name)


@dataclass
class AadTape:
    """A recorded tape (AadTape.java). RANDN / RANDU nodes carry their ordinal in arg_a and their
    stream in arg_b."""
    ops: np.ndarray
    arg_a: np.ndarray
    arg_b: np.ndarray
    constants: np.ndarray
    input_nodes: list
    input_names: list
    recorded_input_values: list
    stream_names: list
    normal_counts: list
    uniform_counts: list
    output_nodes: list
    output_names: list

    def __post_init__(self):
        n = len(self.ops)
        act = np.zeros(n, bool)
        for i in range(n):
            op = AadOp(int(self.ops[i]))
            if op == AadOp.INPUT:
                act[i] = True
            elif op in (AadOp.CONST, AadOp.RANDN, AadOp.RANDU):
                act[i] = False
            elif op in _UNARY:
                act[i] = act[self.arg_a[i]]
            else:
                act[i] = act[self.arg_a[i]] or act[self.arg_b[i]]
        self.active = act

    def size(self) -> int: return len(self.ops)
    def op(self, node: int) -> AadOp: return AadOp(int(self.ops[node]))
    def is_active(self, node: int) -> bool: return bool(self.active[node])
    def input_count(self) -> int: return len(self.input_nodes)
    def input_node(self, index: int) -> int: return self.input_nodes[index]
    def recorded_inputs(self) -> list: return list(self.recorded_input_values)
    def rand_count(self) -> int: return self.normal_counts[0]
    def rand_stream_count(self) -> int: return len(self.stream_names)
    def rand_total(self) -> int: return sum(self.normal_counts) + sum(self.uniform_counts)
    def output_count(self) -> int: return len(self.output_nodes)

    def output_node(self, i: int = 0) -> int:
        return self.output_nodes[i]

    def has_extended_random(self) -> bool:
        """Anything beyond one stream of standard-normal draws (AadTape.java:207-213)."""
        return len(self.stream_names) > 1 or self.uniform_counts[0] > 0

    def __repr__(self) -> str:
        return f"AadTape(nodes={self.size()}, inputs={self.input_names}, randoms={self.rand_count()})"


# ---------------------------------------------------------------------------------------------
# results
# ---------------------------------------------------------------------------------------------

class AadResult:
    """Means over the replayed scenarios (AadResult.java): per output its value, standard error
    and gradient with respect to every input."""

    def __init__(self, output_names, values, stderrs, gradients, input_names, paths: int, seconds: float):
        if not output_names:
            raise ValueError("a result needs at least one output")
        self._out = list(output_names)
        self._val = [float(v) for v in values]
        self._err = [float(v) for v in stderrs]
        self._grad = [list(map(float, g)) for g in gradients]
        self._in = list(input_names)
        self.paths, self.seconds = int(paths), float(seconds)

    def _oi(self, name):
        if name is None:
            return 0
        if name not in self._out:
            raise ValueError(f"unknown output: {name} (have {self._out})")
        return self._out.index(name)

    def _ii(self, name):
        if name not in self._in:
            raise ValueError(f"unknown input: {name}")
        return self._in.index(name)

    def value(self, output: str | None = None) -> float:
        return self._val[self._oi(output)]

    def standard_error(self, output: str | None = None) -> float:
        return self._err[self._oi(output)]

    def gradients(self, output: str | None = None) -> list:
        return list(self._grad[self._oi(output)])

    def gradient(self, a: str, b: str | None = None) -> float:
        """gradient(input) for the primary output, or gradient(output, input)."""
        return self._grad[0][self._ii(a)] if b is None else self._grad[self._oi(a)][self._ii(b)]

    def output_names(self) -> list: return list(self._out)
    def input_names(self) -> list: return list(self._in)
    def output_count(self) -> int: return len(self._out)

    def paths_per_second(self) -> float:
        return self.paths / self.seconds

    def __repr__(self) -> str:
        outs = ", ".join(f"{n}={v}" for n, v in zip(self._out, self._val))
        return f"AadResult({outs}, paths={self.paths})"


class _Accumulator:
    """Combines chunk results weighted by their scenario counts (AadResultAccumulator.java)."""

    def __init__(self, shape: AadResult):
        no, ni = shape.output_count(), len(shape.input_names())
        self.out, self.ins = shape.output_names(), shape.input_names()
        self.vsum, self.sqsum = [0.0] * no, [0.0] * no
        self.known = [True] * no
        self.gsum = [[0.0] * ni for _ in range(no)]
        self.seconds = 0.0

    def add(self, part: AadResult, chunk: int) -> None:
        self.seconds += part.seconds
        for o, name in enumerate(self.out):
            mean = part.value(name)
            self.vsum[o] += mean * chunk
            err = part.standard_error(name)
            if math.isnan(err):
                self.known[o] = False
            elif self.known[o]:
                var = err * err * chunk
                self.sqsum[o] += (chunk - 1 if chunk > 1 else chunk) * var + chunk * mean * mean
            for i, inp in enumerate(self.ins):
                self.gsum[o][i] += part.gradient(name, inp) * chunk

    def result(self, total: int) -> AadResult:
        vals, errs = [], []
        for o in range(len(self.out)):
            v = self.vsum[o] / total
            vals.append(v)
            if self.known[o] and total > 1:
                var = (self.sqsum[o] - total * v * v) / (total - 1)
                errs.append(math.sqrt(max(0.0, var) / total))
            else:
                errs.append(math.nan)
        grads = [[g / total for g in row] for row in self.gsum]
        return AadResult(self.out, vals, errs, grads, self.ins, total, self.seconds)


# ---------------------------------------------------------------------------------------------
# executables
# ---------------------------------------------------------------------------------------------

_ENGINE_ID = {"cuda": 0, "cuda-interp": 1, "cuda-eager": 2}
PROBE_PATHS = 65_536
MIN_CHUNK_PATHS = 4_096


class AadExecutable:
    """A tape compiled by one of the engines (AadExecutable.java, AbstractAadExecutable.java).
    `replay(paths, path_offset, seed)` is one dispatch; `replay_safe` splits a large replay into
    dispatches sized from the measured rate to stay within `max_chunk_seconds`."""

    def __init__(self, engine: str, tape: AadTape, options: AadOptions, device: int = 0):
        self._engine, self._tape, self.options, self.device = engine, tape, options, device
        self.inputs = np.array(tape.recorded_inputs(), np.float64)
        self._rate = 0.0
        env = os.environ.get("NABLATENSOR_MAX_LAUNCH_SECONDS")
        self._max_chunk = float(env) if env else 2.0
        self._closed = False
        eng_opts = options.engine_options_for(engine)
        scratch = int(eng_opts.get("threads" if engine == "cuda-interp" else "bytes", 0) or 0)
        load()
        h = ctypes.c_void_p()
        self._keep = [np.ascontiguousarray(a, np.int32) for a in (tape.ops, tape.arg_a, tape.arg_b)]
        self._cst = np.ascontiguousarray(tape.constants, np.float64)
        self._inn = np.ascontiguousarray(tape.input_nodes if tape.input_nodes else [0], np.int32)
        call("j4b_aad_compile", device, _ENGINE_ID[engine], tape.size(),
             *(k.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)) for k in self._keep),
             self._cst.ctypes.data_as(ctypes.POINTER(ctypes.c_double)), tape.input_count(),
             self._inn.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), tape.output_node(),
             options.precision.value, int(bool(options.adjoints)), scratch, ctypes.byref(h))
        self._h = h.value
        ch, cs, tsl = ctypes.c_int(), ctypes.c_double(), ctypes.c_int64()
        call("j4b_aad_info", self._h, ctypes.byref(ch), ctypes.byref(cs), ctypes.byref(tsl))
        self.channels, self._compile_seconds, self.threads_or_slot = ch.value, cs.value, tsl.value

    # -- the five core methods
    def engine_name(self) -> str:
        return self._engine

    def tape(self) -> AadTape:
        return self._tape

    def set_input(self, name: str, value: float) -> None:
        if name not in self._tape.input_names:
            raise ValueError(f"unknown input: {name}")
        self.inputs[self._tape.input_names.index(name)] = float(value)

    def replay(self, paths: int, path_offset: int = 0, seed: int = 0) -> AadResult:
        self._check_open()
        if paths <= 0:
            raise ValueError("paths must be positive")
        sums = np.zeros(self.channels, np.float64)
        ins = np.ascontiguousarray(self.inputs if len(self.inputs) else [0.0], np.float64)
        t0 = time.perf_counter()
        call("j4b_aad_replay", self._h, ins.ctypes.data_as(ctypes.POINTER(ctypes.c_double)), paths,
             path_offset & 0xFFFFFFFFFFFFFFFF, seed & 0xFFFFFFFFFFFFFFFF,
             sums.ctypes.data_as(ctypes.POINTER(ctypes.c_double)), None)
        seconds = time.perf_counter() - t0
        return self._result(sums, paths, seconds)

    def launch(self, inputs_ptr: int, paths: int, path_offset: int, seed: int, sums_ptr: int, stream=None) -> None:
        """Stream-ordered replay on device buffers (inputs: doubles, sums: `channels` doubles)."""
        self._check_open()
        call("j4b_aad_launch", self._h, inputs_ptr, paths, path_offset & 0xFFFFFFFFFFFFFFFF,
             seed & 0xFFFFFFFFFFFFFFFF, sums_ptr, stream)

    def _result(self, sums: np.ndarray, paths: int, seconds: float) -> AadResult:
        mean = sums[0] / paths
        if paths > 1:
            var = (sums[1] - paths * mean * mean) / (paths - 1)
            err = math.sqrt(max(0.0, var) / paths)
        else:
            err = math.nan
        n_in = self._tape.input_count()
        grads = list(sums[2:2 + n_in] / paths) if self.options.adjoints else [0.0] * n_in
        return AadResult(["value"], [mean], [err], [grads], self._tape.input_names, paths, seconds)

    def close(self) -> None:
        if not self._closed:
            self._closed = True
            if self._h:
                call("j4b_aad_free", self._h)
                self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check_open(self):
        if self._closed:
            raise RuntimeError("executable is closed")

    # -- generated source, compile time
    def source(self) -> str:
        n = ctypes.c_size_t()
        call("j4b_aad_source", self._h, None, 0, ctypes.byref(n))
        buf = ctypes.create_string_buffer(n.value + 1)
        call("j4b_aad_source", self._h, buf, len(buf), ctypes.byref(n))
        return buf.value.decode()

    def compile_seconds(self) -> float:
        return self._compile_seconds

    # -- segmentation (AbstractAadExecutable.java:86-156)
    def max_chunk_seconds(self) -> float:
        return self._max_chunk

    def set_max_chunk_seconds(self, seconds: float) -> None:
        if not seconds > 0.0:
            raise ValueError("maxChunkSeconds must be positive")
        self._max_chunk = seconds

    def measured_paths_per_second(self) -> float:
        return self._rate

    def _observe(self, paths: int, seconds: float) -> None:
        if seconds <= 0.0:
            return
        sample = paths / seconds
        self._rate = sample if self._rate <= 0.0 else 0.5 * (self._rate + sample)

    def _budgeted_chunk(self) -> int:
        if self._rate <= 0.0:
            return PROBE_PATHS
        return max(MIN_CHUNK_PATHS, int(self._rate * self._max_chunk))

    def calibrate(self, seed: int = 0) -> float:
        paths = PROBE_PATHS
        for _ in range(12):
            probe = self.replay(paths, 0, seed)
            self._observe(paths, probe.seconds)
            if probe.seconds >= self._max_chunk * 0.2:
                break
            nxt = self._budgeted_chunk()
            if nxt <= paths:
                break
            paths = min(nxt, paths * 8)
        return self._rate

    def replay_safe(self, total_paths: int, seed: int = 0) -> AadResult:
        if total_paths <= 0:
            raise ValueError("paths must be positive")
        if self._rate <= 0.0:
            self.calibrate(seed)
        acc, done = None, 0
        while done < total_paths:
            chunk = min(self._budgeted_chunk(), total_paths - done)
            part = self.replay(chunk, done, seed)
            if acc is None:
                acc = _Accumulator(part)
            acc.add(part, chunk)
            self._observe(chunk, part.seconds)
            done += chunk
        return acc.result(total_paths)


# ---------------------------------------------------------------------------------------------
# engines
# ---------------------------------------------------------------------------------------------

class AadEngine:
    """One replay backend (AadEngine.java)."""
    name = ""
    priority = 0
    description = ""

    def __init__(self, device: int = 0):
        self.device = device

    def is_available(self) -> bool:
        try:
            import torch
            return torch.cuda.is_available() and torch.cuda.device_count() > self.device
        except Exception:
            return False

    def supports(self, options: AadOptions) -> bool:
        return True

    def describe(self) -> str:
        try:
            import torch
            return f"{self.description} · {torch.cuda.get_device_name(self.device)} · sm_100a"
        except Exception:
            return f"{self.description} · no device"

    def compile(self, tape: AadTape, options: AadOptions | None = None) -> AadExecutable:
        options = options or AadOptions.defaults()
        require_basic_random(tape, self.name)
        require_single_output(tape, self.name)
        return AadExecutable(self.name, tape, options, self.device)


class CudaAadEngine(AadEngine):
    name, priority, description = "cuda", 100, "CUDA"


class CudaInterpEngine(AadEngine):
    name, priority, description = "cuda-interp", 90, "CUDA interpreter (no per-tape compilation)"


class CudaEagerEngine(AadEngine):
    name, priority, description = "cuda-eager", 80, "CUDA eager (one launch per node)"


def require_basic_random(tape: AadTape, engine: str) -> None:
    if tape.has_extended_random():
        raise NotImplementedError(
            f"engine '{engine}' does not yet support rec.randu() or named random streams; use cpu-jit or cpu "
            "for this tape")


def require_single_output(tape: AadTape, engine: str) -> None:
    if tape.output_count() > 1:
        raise NotImplementedError(
            f"engine '{engine}' does not yet support multi-output tapes ({tape.output_names}); use cpu-jit or "
            "cpu for this tape")


ENGINE_PROPERTY = "NABLATENSOR_ENGINE"


class AadEngines:
    """Engine discovery and selection (AadEngines.java): highest priority first."""

    @staticmethod
    def discovered(device: int = 0) -> list:
        return sorted([CudaAadEngine(device), CudaInterpEngine(device), CudaEagerEngine(device)],
                      key=lambda e: -e.priority)

    @staticmethod
    def available(options: AadOptions, device: int = 0) -> list:
        return [e for e in AadEngines.discovered(device) if _usable(e, options)]

    @staticmethod
    def find(name: str, options: AadOptions, device: int = 0):
        for e in AadEngines.discovered(device):
            if e.name.lower() == name.lower() and _usable(e, options):
                return e
        return None

    @staticmethod
    def require(name: str, options: AadOptions, device: int = 0) -> AadEngine:
        e = AadEngines.find(name, options, device)
        if e is None:
            names = ", ".join(x.name for x in AadEngines.available(options, device)) or "(none)"
            raise RuntimeError(f"AAD engine '{name}' is not usable here; available: {names}")
        return e

    @staticmethod
    def select(options: AadOptions, device: int = 0) -> AadEngine:
        requested = os.environ.get(ENGINE_PROPERTY, "").strip()
        if requested:
            return AadEngines.require(requested, options, device)
        usable = AadEngines.available(options, device)
        if not usable:
            names = ", ".join(e.name for e in AadEngines.discovered(device))
            raise RuntimeError(f"no usable AAD engine; discovered: {names}")
        return usable[0]

    @staticmethod
    def compile(tape: AadTape, options: AadOptions | None = None, device: int = 0) -> AadExecutable:
        options = options or AadOptions.defaults()
        return AadEngines.select(options, device).compile(tape, options)


def _usable(engine: AadEngine, options: AadOptions) -> bool:
    try:
        return engine.is_available() and engine.supports(options)
    except Exception:
        return False
