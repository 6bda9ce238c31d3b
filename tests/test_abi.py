"""CPU tests of the C-ABI boundary: the library loads, exports every symbol include/*.h
declares, and rejects bad arguments before touching a device (no compute calls here)."""
import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    inc = os.path.join(ROOT, "include")
    for fname in os.listdir(inc):
        if fname.endswith(".h"):
            text = open(os.path.join(inc, fname)).read()
            names |= set(re.findall(r"^int\s+(j4b_\w+)\s*\(", text, re.M))
    return names


@pytest.fixture(scope="module")
def lib():
    from jax4j_b200 import _lib
    return _lib.load()


def test_library_exports_every_declared_symbol(lib):
    from jax4j_b200 import _lib
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    declared = declared_symbols()
    assert declared, "no declarations parsed"
    missing = declared - exported
    assert not missing, f"declared but not exported: {sorted(missing)}"
    # the ctypes binding covers every declaration
    assert declared <= set(_lib.SIGNATURES), sorted(declared - set(_lib.SIGNATURES))


def test_device_count_never_fails(lib):
    n = ctypes.c_int(-1)
    assert lib.j4b_device_count(ctypes.byref(n)) == 0
    assert n.value >= 0


def test_quant_geometry_checks(lib):
    from jax4j_b200 import _lib
    b = ctypes.c_int64(0)
    assert lib.j4b_quant_bytes(8, 4096, 4096, ctypes.byref(b)) == 0 and b.value == 17825792
    assert lib.j4b_quant_bytes(12, 14336, 4096, ctypes.byref(b)) == 0 and b.value == 33030144
    assert lib.j4b_quant_bytes(2, 10, 64, ctypes.byref(b)) == 0 and b.value == 10 * 2 * 18
    assert lib.j4b_quant_bytes(8, 4, 33, ctypes.byref(b)) == _lib.EINVAL
    assert "block-aligned" in _lib.last_error()
    assert lib.j4b_quant_bytes(14, 4, 512, ctypes.byref(b)) == 0 and b.value == 4 * 2 * 210
    assert lib.j4b_quant_bytes(41, 4, 256, ctypes.byref(b)) == _lib.EUNSUPPORTED
    ids = (ctypes.c_int * 8)()
    n = ctypes.c_int(0)
    assert lib.j4b_quant_supported(ids, 8, ctypes.byref(n)) == 0
    assert sorted(ids[i] for i in range(n.value)) == [2, 8, 12, 14, 42]


def test_invalid_arguments_fail_before_launch(lib):
    from jax4j_b200 import _lib
    with pytest.raises(ValueError, match="not a binary op"):
        _lib.call("j4b_binary", 99, 0, 0, 0, 4, None)
    with pytest.raises(ValueError, match="matmul dimensions must be positive"):
        _lib.call("j4b_matmul", 0, 0, 0, 1, 0, 3, 3, 0, None)
    with pytest.raises(ValueError, match="null quantized weight"):
        _lib.call("j4b_quant_matvec", None, 0, 0, 0, 1, None)
    with pytest.raises(ValueError, match="broadcastTo"):
        src = (ctypes.c_int64 * 1)(3)
        dst = (ctypes.c_int64 * 9)(*([1] * 9))
        _lib.call("j4b_broadcast_to", 0, src, 1, dst, 9, 0, None)


def test_backend_refuses_without_gpu():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from jax4j_b200.backend import B200Backend
    assert B200Backend.is_available() is False
    with pytest.raises(RuntimeError, match="CUDA device"):
        B200Backend(0)


def test_backend_handle_types_construct_without_a_gpu():
    """The handle wrappers the GPU paths return are plain records: constructible and inert here
    (a zero handle frees nothing)."""
    from jax4j_b200.backend import QuantBuffer, QuantPlan
    q = QuantBuffer(0, 8, (2, 32))
    assert q.shape == (2, 32) and q.qtype == 8
    p = QuantPlan(0, (q,), 0)
    assert p.handle == 0
    del p, q
