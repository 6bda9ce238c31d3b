"""ctypes binding of libjax4j_b200.so (declarations in include/jax4j_b200.h).

This is the Python twin of the Java FFM binding a JAX4J engine module would carry: one foreign
function per C-ABI entry point, status codes turned into the exceptions the reference raises
(IllegalArgumentException -> ValueError, UnsupportedOperationException -> NotImplementedError,
driver failures -> RuntimeError). Loading fails loudly when the library has not been built:
there is no fallback path.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("JAX4J_B200_LIB", os.path.join(HERE, "libjax4j_b200.so"))

OK, EINVAL, ENOMEM, ECUDA, EUNSUPPORTED, ENOTINIT, ETIMEOUT = range(7)

Q4_0, Q8_0, Q4_K, Q6_K, Q2_0 = 2, 8, 12, 14, 42
QUANT_NAMES = {Q4_0: "Q4_0", Q8_0: "Q8_0", Q4_K: "Q4_K", Q6_K: "Q6_K", Q2_0: "Q2_0"}
QUANT_BLOCK = {Q4_0: (32, 18), Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210), Q2_0: (128, 34)}

OPS = ["ADD", "SUB", "MUL", "DIV", "MAX", "MIN", "NEG", "EXP", "LOG", "SQRT", "RSQRT", "TANH",
       "SIGMOID", "RELU", "ABS", "SIGN"]
OP = {name: i for i, name in enumerate(OPS)}


class Diagnostics(ctypes.Structure):
    _fields_ = [("dispatches", ctypes.c_uint64), ("allocations", ctypes.c_uint64),
                ("releases", ctypes.c_uint64), ("h2d_bytes", ctypes.c_uint64),
                ("d2h_bytes", ctypes.c_uint64), ("compilations", ctypes.c_uint64)]


class TapeStats(ctypes.Structure):
    _fields_ = [("calls", ctypes.c_int), ("groups", ctypes.c_int), ("folds", ctypes.c_int),
                ("eager_steps", ctypes.c_int), ("fills", ctypes.c_int), ("copies", ctypes.c_int),
                ("launches", ctypes.c_int), ("arena_bytes", ctypes.c_int64)]


_u64 = ctypes.c_uint64
_i64 = ctypes.c_int64
_int = ctypes.c_int
_vp = ctypes.c_void_p
_i64p = ctypes.POINTER(ctypes.c_int64)
_i32p = ctypes.POINTER(ctypes.c_int32)
_f64p = ctypes.POINTER(ctypes.c_double)

# name -> argtypes (every function returns int status)
SIGNATURES = {
    "j4b_init": [ctypes.POINTER(ctypes.c_int), _int],
    "j4b_device_count": [ctypes.POINTER(ctypes.c_int)],
    "j4b_device_name": [_int, ctypes.c_char_p, ctypes.c_size_t],
    "j4b_sm_count": [_int, ctypes.POINTER(ctypes.c_int)],
    "j4b_get_stream": [_int, ctypes.POINTER(_vp)],
    "j4b_sync": [_int],
    "j4b_last_error": [ctypes.c_char_p, ctypes.c_size_t],
    "j4b_get_diagnostics": [ctypes.POINTER(Diagnostics)],
    "j4b_alloc": [_int, ctypes.c_size_t, ctypes.POINTER(_u64)],
    "j4b_free": [_u64],
    "j4b_h2d": [_u64, _vp, ctypes.c_size_t, _vp],
    "j4b_d2h": [_vp, _u64, ctypes.c_size_t, _vp],
    "j4b_d2d": [_u64, _u64, ctypes.c_size_t, _vp],
    "j4b_fill": [_u64, _i64, ctypes.c_float, _vp],
    "j4b_binary": [_int, _u64, _u64, _u64, _i64, _vp],
    "j4b_scalar": [_int, _u64, ctypes.c_double, _u64, _i64, _vp],
    "j4b_unary": [_int, _u64, _u64, _i64, _vp],
    "j4b_transpose": [_u64, _u64, _i64, _i64, _vp],
    "j4b_reduce_sum": [_u64, _i64, _u64, _vp],
    "j4b_reduce_max": [_u64, _i64, _u64, _vp],
    "j4b_reduce_sum_noalloc": [_u64, _i64, _u64, _vp],
    "j4b_sum_axis": [_u64, _i64, _i64, _i64, _u64, _vp],
    "j4b_max_axis": [_u64, _i64, _i64, _i64, _u64, _vp],
    "j4b_argmax_axis": [_u64, _i64, _i64, _i64, _u64, _vp],
    "j4b_max_axis_backward": [_u64, _u64, _i64, _i64, _i64, _u64, _vp],
    "j4b_broadcast_to": [_u64, _i64p, _int, _i64p, _int, _u64, _vp],
    "j4b_reindex": [_u64, _i64, _u64, _i64, _u64, _vp],
    "j4b_scatter_add": [_u64, _i64, _u64, _i64, _u64, _vp],
    "j4b_relu_backward": [_u64, _u64, _u64, _i64, _vp],
    "j4b_random_uniform": [_i64, _i64, _u64, _i64, _vp],
    "j4b_random_normal": [_i64, _i64, _u64, _i64, _vp],
    "j4b_matmul": [_u64, _u64, _u64, _i64, _i64, _i64, _i64, _int, _vp],
    "j4b_conv2d": [_u64, _u64, _u64, _i64, _int, _int, _int, _int, _int, _int, _int, _int, _vp],
    "j4b_conv2d_grad_input": [_u64, _u64, _u64, _i64, _int, _int, _int, _int, _int, _int, _int, _int, _vp],
    "j4b_conv2d_grad_weight": [_u64, _u64, _u64, _i64, _int, _int, _int, _int, _int, _int, _int, _int, _vp],
    "j4b_quant_supported": [ctypes.POINTER(ctypes.c_int), _int, ctypes.POINTER(ctypes.c_int)],
    "j4b_quant_bytes": [_int, _i64, _i64, _i64p],
    "j4b_quant_upload": [_int, _vp, ctypes.c_size_t, _int, _i64, _i64, ctypes.POINTER(_vp)],
    "j4b_quant_upload_device": [_int, _u64, ctypes.c_size_t, _int, _i64, _i64,
                                ctypes.POINTER(_vp)],
    "j4b_quant_free": [_vp],
    "j4b_quant_shape": [_vp, ctypes.POINTER(ctypes.c_int), _i64p, _i64p],
    "j4b_quant_matvec": [_vp, _u64, _u64, _u64, _i64, _vp],
    "j4b_quant_matvec_host": [_vp, _vp, _i64, _vp, _vp],
    "j4b_quant_gather_row": [_vp, _i64, _u64, _vp],
    "j4b_quantize": [_int, _u64, _i64, _i64, _u64, _vp],
    "j4b_quant_gemm": [_vp, _u64, _u64, _i64, _int, _vp],
    "j4b_rmsnorm": [_u64, _u64, ctypes.c_float, _i64, _i64, _u64, _vp],
    "j4b_rope_kv": [_u64, _i64, _i64, _i64, _i64, _i64, ctypes.c_double, _u64, _u64, _u64, _i64, _vp],
    "j4b_attention_decode": [_u64, _u64, _u64, _i64, _i64, _i64, _i64, _i64, _u64, _vp],
    "j4b_attention_prefill": [_u64, _u64, _u64, _i64, _i64, _i64, _i64, _i64, _u64, _vp],
    "j4b_swiglu": [_u64, _i64, _i64, _u64, _vp],
    "j4b_peer_alloc": [_int, ctypes.c_size_t, ctypes.POINTER(_u64), ctypes.c_char_p],
    "j4b_peer_open": [_int, ctypes.c_char_p, ctypes.POINTER(_u64)],
    "j4b_peer_close": [_u64],
    "j4b_peer_free": [_u64],
    "j4b_peer_group_create": [_int, _int, _int, ctypes.POINTER(_u64), ctypes.c_size_t,
                              ctypes.POINTER(_vp)],
    "j4b_peer_group_free": [_vp],
    "j4b_peer_status": [_vp, ctypes.POINTER(ctypes.c_int)],
    "j4b_quant_matvec_allgather": [_vp, _u64, _u64, _u64, _i64, _vp, _int, _vp],
    "j4b_quant_matvec_allgather_host": [_vp, _vp, _i64, _vp, _vp, _int, _vp],
    "j4b_quant_matvec_host_plan": [_vp, _vp, _i64, _vp, _vp, _int, ctypes.POINTER(_vp)],
    "j4b_quant_matvec_host_run": [_vp, _vp],
    "j4b_quant_matvec_host_plan_free": [_vp],
    "j4b_peer_allreduce": [_vp, _int, _u64, _i64, _u64, _vp],
    "j4b_tape_compile": [_int, _i64p, ctypes.c_size_t, ctypes.POINTER(_vp)],
    "j4b_tape_launch": [_vp, ctypes.POINTER(_u64), _int, ctypes.POINTER(_u64), _int, _vp],
    "j4b_tape_free": [_vp],
    "j4b_tape_info": [_vp, ctypes.POINTER(TapeStats)],
    "j4b_tape_dryrun": [_i64p, ctypes.c_size_t, ctypes.POINTER(TapeStats), ctypes.c_char_p,
                        ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t)],
    "j4b_tape_source": [_vp, _int, ctypes.c_char_p, ctypes.c_size_t,
                        ctypes.POINTER(ctypes.c_size_t)],
    "j4b_aad_compile": [_int, _int, _int, _i32p, _i32p, _i32p, _f64p, _int, _i32p, _int, _int, _int,
                        _i64, ctypes.POINTER(_vp)],
    "j4b_aad_replay": [_vp, _f64p, _u64, _u64, _u64, _f64p, _vp],
    "j4b_aad_launch": [_vp, _u64, _u64, _u64, _u64, _u64, _vp],
    "j4b_aad_info": [_vp, ctypes.POINTER(ctypes.c_int), _f64p, _i64p],
    "j4b_aad_source": [_vp, ctypes.c_char_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t)],
    "j4b_aad_free": [_vp],
    "j4b_aad_dryrun": [_int, _i32p, _i32p, _i32p, _f64p, _int, _i32p, _int, _int, _int,
                       ctypes.c_char_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t)],
}

_lib = None


def load():
    """Loads the engine library; raises if it has not been built (no fallback exists)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(
            f"jax4j_b200 engine library not found at {LIB_PATH}; build it with "
            "`python -m jax4j_b200.build` (the engine has no CPU fallback)")
    lib = ctypes.CDLL(LIB_PATH)
    for name, argtypes in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = ctypes.c_int
    _lib = lib
    return lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    load().j4b_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(status: int, what: str = "") -> None:
    if status == OK:
        return
    msg = last_error() or what
    if status == EINVAL:
        raise ValueError(msg)
    if status == EUNSUPPORTED:
        raise NotImplementedError(msg)
    if status == ENOMEM:
        raise MemoryError(msg)
    if status == ETIMEOUT:
        raise TimeoutError(msg)
    raise RuntimeError(msg)


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args), name)


def diagnostics() -> dict:
    d = Diagnostics()
    call("j4b_get_diagnostics", ctypes.byref(d))
    return {name: int(getattr(d, name)) for name, _ in Diagnostics._fields_}


def exported_symbols() -> list[str]:
    return list(SIGNATURES)


def tape_dryrun(words) -> tuple[dict, str]:
    """Plans a serialised tape and compiles its kernels with NVRTC, without a device: returns the
    plan statistics and the generated CUDA source (j4b_tape_dryrun)."""
    import numpy as np
    w = np.ascontiguousarray(words, dtype=np.int64)
    st = TapeStats()
    n = ctypes.c_size_t(0)
    call("j4b_tape_dryrun", w.ctypes.data_as(_i64p), w.size, ctypes.byref(st), None, 0,
         ctypes.byref(n))
    buf = ctypes.create_string_buffer(n.value + 1)
    call("j4b_tape_dryrun", w.ctypes.data_as(_i64p), w.size, ctypes.byref(st), buf, n.value + 1,
         ctypes.byref(n))
    stats = {name: int(getattr(st, name)) for name, _ in TapeStats._fields_}
    return stats, buf.value.decode()
