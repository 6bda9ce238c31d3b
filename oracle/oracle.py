"""TEST INFRASTRUCTURE ONLY -- numpy/ctypes front of the C oracle (oracle.c).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline legs may import this
module; the engine never does. Every function restates the reference's jax4j-core CPU path
(citations live beside the C functions in oracle.c).
"""
from __future__ import annotations

import ctypes
import os
import struct
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle_j4b.so")
_lib = None

Q4_0, Q8_0, Q4_K, Q6_K, Q2_0 = 2, 8, 12, 14, 42
BLOCK = {Q4_0: (32, 18), Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210), Q2_0: (128, 34)}

OPS = ["ADD", "SUB", "MUL", "DIV", "MAX", "MIN", "NEG", "EXP", "LOG", "SQRT", "RSQRT", "TANH",
       "SIGMOID", "RELU", "ABS", "SIGN"]
OP = {name: i for i, name in enumerate(OPS)}


def build() -> str:
    """Compiles liboracle_j4b.so with the committed Makefile if it is missing or stale."""
    src = os.path.join(_HERE, "oracle.c")
    if (not os.path.exists(_LIB_PATH)
            or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src)):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        _lib = ctypes.CDLL(_LIB_PATH)
        _declare(_lib)
    return _lib


_f32p = ctypes.POINTER(ctypes.c_float)
_f64p = ctypes.POINTER(ctypes.c_double)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_i32p = ctypes.POINTER(ctypes.c_int32)
_i64p = ctypes.POINTER(ctypes.c_int64)
_i64 = ctypes.c_int64


def _declare(L):
    L.j4o_mix64.restype = ctypes.c_uint64
    L.j4o_mix64.argtypes = [ctypes.c_uint64]
    L.j4o_random_uniform.argtypes = [_i64, _i64, _i64, _f32p]
    L.j4o_random_normal.argtypes = [_i64, _i64, _i64, _f32p]
    L.j4o_prng_split.argtypes = [_i64, _i64, ctypes.c_int, _i64p]
    L.j4o_half_to_float.restype = ctypes.c_float
    L.j4o_half_to_float.argtypes = [ctypes.c_uint32]
    L.j4o_float_to_half.restype = ctypes.c_uint16
    L.j4o_float_to_half.argtypes = [ctypes.c_float]
    L.j4o_quant_row_bytes.restype = _i64
    L.j4o_quant_row_bytes.argtypes = [ctypes.c_int, _i64]
    L.j4o_quantize.argtypes = [ctypes.c_int, _f32p, _i64, _i64, _u8p]
    L.j4o_gather_row.argtypes = [ctypes.c_int, _u8p, _i64, _i64, _i64, _f32p]
    L.j4o_quant_matvec.argtypes = [ctypes.c_int, _u8p, _i64, _i64, _f32p, _i64, _f32p]
    L.j4o_quant_matvec_f64.argtypes = [ctypes.c_int, _u8p, _i64, _i64, _f32p, _i64, _f64p]
    L.j4o_apply_binary.restype = ctypes.c_float
    L.j4o_apply_binary.argtypes = [ctypes.c_int, ctypes.c_float, ctypes.c_float]
    L.j4o_apply_unary.restype = ctypes.c_float
    L.j4o_apply_unary.argtypes = [ctypes.c_int, ctypes.c_float]
    L.j4o_binary.argtypes = [ctypes.c_int, _f32p, _f32p, _i64, _f32p]
    L.j4o_scalar.argtypes = [ctypes.c_int, _f32p, ctypes.c_double, _i64, _f32p]
    L.j4o_unary.argtypes = [ctypes.c_int, _f32p, _i64, _f32p]
    L.j4o_transpose.argtypes = [_f32p, _i64, _i64, _f32p]
    L.j4o_matmul.argtypes = [_f32p, _f32p, _i64, _i64, _i64, _f32p]
    L.j4o_batched_matmul.argtypes = [_f32p, _f32p, _i64, _i64, _i64, _i64, _f32p]
    L.j4o_reduce_sum.restype = ctypes.c_float
    L.j4o_reduce_sum.argtypes = [_f32p, _i64]
    L.j4o_reduce_max.restype = ctypes.c_float
    L.j4o_reduce_max.argtypes = [_f32p, _i64]
    for name in ("j4o_sum_axis", "j4o_max_axis", "j4o_argmax_axis"):
        getattr(L, name).argtypes = [_f32p, _i64, _i64, _i64, _f32p]
    L.j4o_max_axis_backward.argtypes = [_f32p, _f32p, _i64, _i64, _i64, _f32p]
    L.j4o_broadcast_to.argtypes = [_f32p, _i64p, ctypes.c_int, _i64p, ctypes.c_int, _f32p]
    L.j4o_reindex.argtypes = [_f32p, _i64, _i32p, _i64, _f32p]
    L.j4o_scatter_add.argtypes = [_f32p, _i64, _i32p, _i64, _f32p]
    L.j4o_relu_backward.argtypes = [_f32p, _f32p, _i64, _f32p]
    L.j4o_fused.argtypes = [_i32p, ctypes.c_int, ctypes.POINTER(_f32p), ctypes.c_int, _i64,
                            _f32p]
    for name in ("j4o_conv2d", "j4o_conv2d_grad_input", "j4o_conv2d_grad_weight"):
        getattr(L, name).argtypes = [_f32p, _f32p, _i64] + [ctypes.c_int] * 7 + [_f32p]
    L.j4o_aad_replay.argtypes = [ctypes.c_int, _i32p, _i32p, _i32p, _f64p, _f64p, ctypes.c_int, _i32p,
                                 ctypes.c_int, _i32p, ctypes.c_int, ctypes.c_int, _i64, _i64, _i64,
                                 _f64p, _f64p, _f64p]
    L.j4o_philox2x32_10.argtypes = [ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,
                                    ctypes.POINTER(ctypes.c_uint32), ctypes.POINTER(ctypes.c_uint32)]


def _p(a, t=_f32p):
    return a.ctypes.data_as(t)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


# ---- PRNG -------------------------------------------------------------------------------------

def random_uniform(seed: int, counter: int, n: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().j4o_random_uniform(seed, counter, n, _p(out))
    return out


def random_normal(seed: int, counter: int, n: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().j4o_random_normal(seed, counter, n, _p(out))
    return out


def prng_split(seed: int, counter: int, count: int) -> list[int]:
    out = np.empty(count, np.int64)
    lib().j4o_prng_split(seed, counter, count, _p(out, _i64p))
    return [int(v) for v in out]


def half_to_float(bits: int) -> float:
    return lib().j4o_half_to_float(bits)


def float_to_half(v: float) -> int:
    return lib().j4o_float_to_half(v)


# ---- quant ------------------------------------------------------------------------------------

def quant_row_bytes(qtype: int, cols: int) -> int:
    return lib().j4o_quant_row_bytes(qtype, cols)


def quantize(qtype: int, w: np.ndarray) -> np.ndarray:
    w = _f32(w)
    rows, cols = w.shape
    rb = quant_row_bytes(qtype, cols)
    if rb < 0:
        raise ValueError("bad quant geometry")
    out = np.empty(rows * rb, np.uint8)
    if lib().j4o_quantize(qtype, _p(w), rows, cols, _p(out, _u8p)) != 0:
        raise ValueError("quantize failed")
    return out


def gather_row(qtype: int, blob: np.ndarray, rows: int, cols: int, row: int) -> np.ndarray:
    out = np.empty(cols, np.float32)
    blob = np.ascontiguousarray(blob, np.uint8)
    if lib().j4o_gather_row(qtype, _p(blob, _u8p), rows, cols, row, _p(out)) != 0:
        raise ValueError("gather_row failed")
    return out


def dequantize(qtype: int, blob: np.ndarray, rows: int, cols: int) -> np.ndarray:
    return np.stack([gather_row(qtype, blob, rows, cols, r) for r in range(rows)])


def quant_matvec(qtype: int, blob: np.ndarray, rows: int, cols: int, x: np.ndarray) -> np.ndarray:
    """Float-sequential reference order; x is [batch, cols] -> y [batch, rows]."""
    x = _f32(x).reshape(-1, cols)
    y = np.empty((x.shape[0], rows), np.float32)
    blob = np.ascontiguousarray(blob, np.uint8)
    if lib().j4o_quant_matvec(qtype, _p(blob, _u8p), rows, cols, _p(x), x.shape[0], _p(y)):
        raise ValueError("quant_matvec failed")
    return y


def quant_matvec_f64(qtype: int, blob: np.ndarray, rows: int, cols: int,
                     x: np.ndarray) -> np.ndarray:
    x = _f32(x).reshape(-1, cols)
    y = np.empty((x.shape[0], rows), np.float64)
    blob = np.ascontiguousarray(blob, np.uint8)
    if lib().j4o_quant_matvec_f64(qtype, _p(blob, _u8p), rows, cols, _p(x), x.shape[0],
                                  _p(y, _f64p)):
        raise ValueError("quant_matvec_f64 failed")
    return y


# ---- CpuBackend primitives -------------------------------------------------------------------

def binary(op: str, a, b):
    a, b = _f32(a), _f32(b)
    if a.size != b.size:
        raise ValueError(f"shape mismatch: {a.shape} vs {b.shape}")
    out = np.empty_like(a)
    lib().j4o_binary(OP[op], _p(a), _p(b), a.size, _p(out))
    return out


def scalar(op: str, a, value: float):
    a = _f32(a)
    out = np.empty_like(a)
    lib().j4o_scalar(OP[op], _p(a), float(value), a.size, _p(out))
    return out


def unary(op: str, a):
    a = _f32(a)
    out = np.empty_like(a)
    lib().j4o_unary(OP[op], _p(a), a.size, _p(out))
    return out


def transpose(a):
    a = _f32(a)
    r, c = a.shape
    out = np.empty((c, r), np.float32)
    lib().j4o_transpose(_p(a), r, c, _p(out))
    return out


def matmul(a, b):
    a, b = _f32(a), _f32(b)
    m, k = a.shape
    k2, n = b.shape
    if k != k2:
        raise ValueError("incompatible matmul shapes")
    out = np.empty((m, n), np.float32)
    lib().j4o_matmul(_p(a), _p(b), m, k, n, _p(out))
    return out


def batched_matmul(a, b):
    a, b = _f32(a), _f32(b)
    bt, m, k = a.shape
    _, _, n = b.shape
    out = np.empty((bt, m, n), np.float32)
    lib().j4o_batched_matmul(_p(a), _p(b), bt, m, k, n, _p(out))
    return out


def reduce_sum(a):
    a = _f32(a)
    return np.array([lib().j4o_reduce_sum(_p(a), a.size)], np.float32)


def reduce_max(a):
    a = _f32(a)
    return np.array([lib().j4o_reduce_max(_p(a), a.size)], np.float32)


def _axis_split(shape, axis):
    outer = int(np.prod(shape[:axis], dtype=np.int64))
    inner = int(np.prod(shape[axis + 1:], dtype=np.int64))
    return outer, shape[axis], inner


def _axis_out_shape(shape, axis, keep):
    return tuple(1 if i == axis else d for i, d in enumerate(shape)) if keep else \
        tuple(d for i, d in enumerate(shape) if i != axis)


def sum_axis(a, axis: int, keep: bool = False):
    a = _f32(a)
    o, n, i = _axis_split(a.shape, axis)
    out = np.empty(o * i, np.float32)
    lib().j4o_sum_axis(_p(a), o, n, i, _p(out))
    return out.reshape(_axis_out_shape(a.shape, axis, keep))


def max_axis(a, axis: int, keep: bool = False):
    a = _f32(a)
    o, n, i = _axis_split(a.shape, axis)
    out = np.empty(o * i, np.float32)
    lib().j4o_max_axis(_p(a), o, n, i, _p(out))
    return out.reshape(_axis_out_shape(a.shape, axis, keep))


def argmax_axis(a, axis: int):
    a = _f32(a)
    o, n, i = _axis_split(a.shape, axis)
    out = np.empty(o * i, np.float32)
    lib().j4o_argmax_axis(_p(a), o, n, i, _p(out))
    return out.reshape(_axis_out_shape(a.shape, axis, False))


def max_axis_backward(up, a, axis: int):
    a, up = _f32(a), _f32(up)
    o, n, i = _axis_split(a.shape, axis)
    out = np.empty_like(a)
    lib().j4o_max_axis_backward(_p(up), _p(a), o, n, i, _p(out))
    return out


def broadcast_to(a, target):
    a = _f32(a)
    sd = np.array(a.shape if a.ndim else (1,), np.int64)
    td = np.array(target, np.int64)
    out = np.empty(tuple(target), np.float32)
    lib().j4o_broadcast_to(_p(a), _p(sd, _i64p), len(sd), _p(td, _i64p), len(td), _p(out))
    return out


def reindex(a, target, indices):
    a = _f32(a)
    m = np.ascontiguousarray(indices, np.int32)
    out = np.empty(int(np.prod(target)), np.float32)
    if lib().j4o_reindex(_p(a), a.size, _p(m, _i32p), m.size, _p(out)):
        raise ValueError("index out of bounds")
    return out.reshape(target)


def scatter_add(a, target, indices):
    a = _f32(a)
    m = np.ascontiguousarray(indices, np.int32)
    n = int(np.prod(target))
    out = np.empty(n, np.float32)
    if lib().j4o_scatter_add(_p(a), a.size, _p(m, _i32p), n, _p(out)):
        raise ValueError("index out of bounds")
    return out.reshape(target)


def relu_backward(up, a):
    a, up = _f32(a), _f32(up)
    out = np.empty_like(a)
    lib().j4o_relu_backward(_p(up), _p(a), a.size, _p(out))
    return out


def fused(prog: list[int], inputs: list[np.ndarray]):
    """Evaluates a postfix expression program (see oracle.h) per element."""
    ins = [_f32(x) for x in inputs]
    n = ins[0].size
    arr = (_f32p * len(ins))(*[_p(x) for x in ins])
    p = np.ascontiguousarray(prog, np.int32)
    out = np.empty(n, np.float32)
    if lib().j4o_fused(_p(p, _i32p), len(p), arr, len(ins), n, _p(out)):
        raise ValueError("bad fused program")
    return out.reshape(ins[0].shape)


def scalar_words(value: float) -> list[int]:
    """Splits a double into the two int32 words a scalar op carries in a postfix program."""
    lo, hi = struct.unpack("<ii", struct.pack("<d", value))
    return [lo, hi]


# ---- scalar-AAD Monte-Carlo replay (the CPU engine, ScalarReplay) ----

def philox2x32_10(c0: int, c1: int, key: int = 0x1BD11BDA) -> tuple[int, int]:
    o0, o1 = ctypes.c_uint32(), ctypes.c_uint32()
    lib().j4o_philox2x32_10(c0 & 0xFFFFFFFF, c1 & 0xFFFFFFFF, key & 0xFFFFFFFF, ctypes.byref(o0),
                            ctypes.byref(o1))
    return o0.value, o1.value


def aad_replay(ops, arg_a, arg_b, constants, inputs, input_nodes, output_nodes, n_streams, paths,
               path_offset, seed, adjoints=True, threads=1):
    """Sums over scenarios [path_offset, path_offset + paths): per output the value sum and the
    value^2 sum, and [output][input] the adjoint sums. With threads > 1 the range is split into
    contiguous runs as ScalarReplay.runParallel does (ctypes releases the GIL during each run)."""
    ops, a, b = (np.ascontiguousarray(v, np.int32) for v in (ops, arg_a, arg_b))
    cst = np.ascontiguousarray(constants, np.float64)
    ins = np.ascontiguousarray(inputs if len(inputs) else [0.0], np.float64)
    inn = np.ascontiguousarray(input_nodes if len(input_nodes) else [0], np.int32)
    outn = np.ascontiguousarray(output_nodes, np.int32)
    n_in, n_out = len(input_nodes), len(outn)

    def run(frm, count):
        v, sq = np.zeros(n_out), np.zeros(n_out)
        g = np.zeros(max(1, n_out * n_in))
        rc = lib().j4o_aad_replay(len(ops), _p(ops, _i32p), _p(a, _i32p), _p(b, _i32p), _p(cst, _f64p),
                                  _p(ins, _f64p), n_in, _p(inn, _i32p), n_out, _p(outn, _i32p),
                                  n_streams, int(bool(adjoints)), frm, count, seed & 0xFFFFFFFFFFFFFFFF
                                  if seed < 2 ** 63 else seed - 2 ** 64, _p(v, _f64p), _p(sq, _f64p),
                                  _p(g, _f64p))
        if rc:
            raise ValueError("invalid tape")
        return v, sq, g[:n_out * n_in].reshape(n_out, n_in)

    threads = max(1, min(threads, paths))
    if threads == 1:
        return run(path_offset, paths)
    from concurrent.futures import ThreadPoolExecutor
    each, extra = divmod(paths, threads)
    runs, cur = [], path_offset
    for t in range(threads):
        c = each + (1 if t < extra else 0)
        runs.append((cur, c))
        cur += c
    with ThreadPoolExecutor(threads) as ex:
        parts = list(ex.map(lambda r: run(*r), runs))
    return tuple(sum(p[i] for p in parts) for i in range(3))


# ---- conv2d (CpuBackend.conv2d / conv2dGradInput / conv2dGradWeight) ----

def _conv_out(spec):
    c, h, w, o, k, s, p = spec
    return o * ((h + 2 * p - k) // s + 1) * ((w + 2 * p - k) // s + 1)


def conv2d(x, w, spec):
    """spec = (in_c, in_h, in_w, out_c, kernel, stride, pad); x [batch, in_c*in_h*in_w]."""
    x, w = _f32(x), _f32(w)
    out = np.empty((x.shape[0], _conv_out(spec)), np.float32)
    if lib().j4o_conv2d(_p(x), _p(w), x.shape[0], *spec, _p(out)):
        raise ValueError("invalid conv spec")
    return out


def conv2d_grad_input(up, w, spec):
    up, w = _f32(up), _f32(w)
    c, h, wd = spec[0], spec[1], spec[2]
    out = np.empty((up.shape[0], c * h * wd), np.float32)
    if lib().j4o_conv2d_grad_input(_p(up), _p(w), up.shape[0], *spec, _p(out)):
        raise ValueError("invalid conv spec")
    return out


def conv2d_grad_weight(x, up, spec):
    x, up = _f32(x), _f32(up)
    out = np.empty((spec[3], spec[0] * spec[4] * spec[4]), np.float32)
    if lib().j4o_conv2d_grad_weight(_p(x), _p(up), x.shape[0], *spec, _p(out)):
        raise ValueError("invalid conv spec")
    return out
