"""B200Backend: the engine SPI (ComputeBackend + QuantizedOps) over the C ABI.

Mirrors core/tensor/spi/ComputeBackend.java:36-296 and QuantizedOps.java:19-34 method for
method (snake_case names), with the reference's argument checks and messages, so code written
against the reference's SPI reads the same here. Every numerical call is one C-ABI entry point of
libjax4j_b200.so; device memory and streams come from PyTorch (plumbing only), and nothing falls
back to the CPU: without a CUDA device and the built library, construction fails.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import numpy as np
import torch

from . import _lib
from ._lib import OP, QUANT_BLOCK, QUANT_NAMES, call


def _prod(dims) -> int:
    n = 1
    for d in dims:
        n *= int(d)
    return n


CUDA_STREAM_LEGACY = 1  # cudaStreamLegacy


def torch_stream(device=None) -> int:
    """Handle of PyTorch's current stream, in the C ABI's convention."""
    s = torch.cuda.current_stream(device).cuda_stream
    return s if s else CUDA_STREAM_LEGACY


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


@dataclass(eq=False)
class DeviceBuffer:
    """DeviceBuffer (core/tensor/spi/DeviceBuffer.java:26-33): shape + f32 device storage."""
    tensor: torch.Tensor
    shape: tuple
    dtype: str = "F32"
    released: bool = field(default=False)

    @property
    def ptr(self) -> int:
        if self.released:
            raise ValueError("buffer has been released")
        return self.tensor.data_ptr()

    @property
    def size(self) -> int:
        return _prod(self.shape)


class QuantPlan:
    """A recorded host-buffer quantMatvec (j4b_quant_matvec_host_plan); `run` replays it."""

    def __init__(self, handle: int, keep: tuple, default_stream: int):
        self.handle, self._keep, self._stream = handle, keep, default_stream

    @staticmethod
    def make(w, x_host, y_host, batch: int, group_handle, channel: int, stream: int) -> "QuantPlan":
        h = ctypes.c_void_p()
        call("j4b_quant_matvec_host_plan", ctypes.c_void_p(w.handle), x_host.data_ptr(), batch, y_host.data_ptr(),
             group_handle, channel, ctypes.byref(h))
        return QuantPlan(h.value, (w, x_host, y_host), stream)

    def run(self, stream: int | None = None) -> None:
        call("j4b_quant_matvec_host_run", self.handle, self._stream if stream is None else stream)

    def __del__(self):
        if getattr(self, "handle", None) and _lib._lib is not None:
            _lib.load().j4b_quant_matvec_host_plan_free(ctypes.c_void_p(self.handle))
            self.handle = None


@dataclass(eq=False)
class QuantBuffer:
    """Opaque quantized matrix (the CpuQuantBuffer role, CpuQuantBuffer.java:10-38)."""
    handle: int
    qtype: int
    shape: tuple
    dtype: str = "F32"

    def __del__(self):
        if self.handle and _lib._lib is not None:
            _lib.load().j4b_quant_free(ctypes.c_void_p(self.handle))
            self.handle = 0


class TapeHandle:
    """A compiled tape on one device."""

    def __init__(self, backend: "B200Backend", tape):
        words = np.ascontiguousarray(tape.serialize(), dtype=np.int64)
        h = ctypes.c_void_p()
        call("j4b_tape_compile", backend.device, words.ctypes.data_as(_lib._i64p), words.size,
             ctypes.byref(h))
        self.handle = h
        self.backend = backend
        self.in_shapes = [tuple(tape.shapes[i]) for i in tape.inputs]
        self.out_shapes = [tuple(tape.shapes[o]) for o in tape.outputs]

    def stats(self) -> dict:
        st = _lib.TapeStats()
        call("j4b_tape_info", self.handle, ctypes.byref(st))
        return {name: int(getattr(st, name)) for name, _ in _lib.TapeStats._fields_}

    def source(self, group: int) -> str:
        n = ctypes.c_size_t(0)
        call("j4b_tape_source", self.handle, group, None, 0, ctypes.byref(n))
        buf = ctypes.create_string_buffer(n.value + 1)
        call("j4b_tape_source", self.handle, group, buf, n.value + 1, ctypes.byref(n))
        return buf.value.decode()

    def launch(self, in_ptrs: list, out_ptrs: list, stream: int) -> None:
        ins = (ctypes.c_uint64 * max(len(in_ptrs), 1))(*in_ptrs)
        outs = (ctypes.c_uint64 * max(len(out_ptrs), 1))(*out_ptrs)
        call("j4b_tape_launch", self.handle, ins, len(in_ptrs), outs, len(out_ptrs), stream)

    def run(self, buffers: list) -> list:
        for b, s in zip(buffers, self.in_shapes):
            if tuple(b.shape) != s:
                raise ValueError(f"tape input shape {b.shape} does not match the recorded {s}")
        outs = [self.backend._new(s) for s in self.out_shapes]
        self.launch([b.ptr for b in buffers], [o.ptr for o in outs], self.backend.stream)
        return outs

    def __del__(self):
        if getattr(self, "handle", None) and _lib._lib is not None:
            _lib.load().j4b_tape_free(self.handle)
            self.handle = None


class B200Backend:
    """The sm_100a engine behind name() == "cuda" (BackendRegistry selects it by name)."""
    executes_tapes = True

    def __init__(self, device: int = 0):
        if not torch.cuda.is_available():
            raise RuntimeError("B200Backend requires a CUDA device")
        _lib.load()
        self.device = device
        dev = (ctypes.c_int * 1)(device)
        call("j4b_init", dev, 1)
        self._torch_device = torch.device("cuda", device)

    # ---- identity (ComputeBackend.java:38-46) ----
    def name(self) -> str:
        return "cuda"

    def device_type(self) -> str:
        return "CUDA"

    @staticmethod
    def is_available() -> bool:
        """Never raises (CudaBackend.isAvailable contract, CudaBackend.java:427-434)."""
        try:
            lib = _lib.load()
            n = ctypes.c_int(0)
            return lib.j4b_device_count(ctypes.byref(n)) == 0 and n.value > 0
        except Exception:
            return False

    def priority(self) -> int:
        return 200

    # ---- plumbing ----
    @property
    def stream(self) -> int:
        """PyTorch's current stream; its default stream (handle 0) is passed as cudaStreamLegacy,
        since a NULL stream selects the engine's own stream in the C ABI."""
        return torch_stream(self._torch_device)

    def _new(self, shape) -> DeviceBuffer:
        t = torch.empty(max(_prod(shape), 1), dtype=torch.float32, device=self._torch_device)
        return DeviceBuffer(t, tuple(int(d) for d in shape))

    def wrap(self, t: torch.Tensor) -> DeviceBuffer:
        if t.dtype != torch.float32 or not t.is_cuda:
            raise ValueError("wrap expects a CUDA float32 tensor")
        t = t.contiguous()
        return DeviceBuffer(t.reshape(-1), tuple(t.shape))

    # ---- upload / download (ComputeBackend.java:48, 87) ----
    def upload(self, data, shape, dtype: str = "F32") -> DeviceBuffer:
        arr = np.ascontiguousarray(np.asarray(data, dtype=np.float32).reshape(-1))
        if arr.size != _prod(shape):
            raise ValueError("Upload length does not match shape")
        if dtype != "F32":
            raise NotImplementedError(f"CUDA tensor upload supports F32 only, got {dtype}")
        out = self._new(shape)
        call("j4b_h2d", out.ptr, arr.ctypes.data_as(ctypes.c_void_p), arr.nbytes, self.stream)
        torch.cuda.current_stream(self._torch_device).synchronize()
        return out

    def download(self, buf: DeviceBuffer) -> np.ndarray:
        out = np.empty(buf.size, np.float32)
        call("j4b_d2h", out.ctypes.data_as(ctypes.c_void_p), buf.ptr, out.nbytes, self.stream)
        return out.reshape(buf.shape)

    def full(self, value: float, shape, dtype: str = "F32") -> DeviceBuffer:
        out = self._new(shape)
        call("j4b_fill", out.ptr, out.size, float(value), self.stream)
        return out

    def random_uniform(self, seed: int, counter: int, shape) -> DeviceBuffer:
        out = self._new(shape)
        call("j4b_random_uniform", seed, counter, out.ptr, out.size, self.stream)
        return out

    def random_normal(self, seed: int, counter: int, shape) -> DeviceBuffer:
        out = self._new(shape)
        call("j4b_random_normal", seed, counter, out.ptr, out.size, self.stream)
        return out

    # ---- elementwise (ComputeBackend.java:89-93) ----
    def binary(self, op: str, a: DeviceBuffer, b: DeviceBuffer) -> DeviceBuffer:
        if a.size != b.size:
            raise ValueError(f"shape mismatch: {a.shape} vs {b.shape}")
        out = self._new(a.shape)
        call("j4b_binary", OP[op], a.ptr, b.ptr, out.ptr, a.size, self.stream)
        return out

    def scalar(self, op: str, a: DeviceBuffer, value: float) -> DeviceBuffer:
        out = self._new(a.shape)
        call("j4b_scalar", OP[op], a.ptr, float(value), out.ptr, a.size, self.stream)
        return out

    def unary(self, op: str, a: DeviceBuffer) -> DeviceBuffer:
        out = self._new(a.shape)
        call("j4b_unary", OP[op], a.ptr, out.ptr, a.size, self.stream)
        return out

    def relu_backward(self, upstream: DeviceBuffer, inp: DeviceBuffer) -> DeviceBuffer:
        out = self._new(upstream.shape)
        call("j4b_relu_backward", upstream.ptr, inp.ptr, out.ptr, upstream.size, self.stream)
        return out

    # ---- movement / contraction ----
    def transpose(self, a: DeviceBuffer) -> DeviceBuffer:
        if len(a.shape) != 2:
            raise ValueError(f"transpose requires a rank-2 tensor, got {a.shape}")
        r, c = a.shape
        out = self._new((c, r))
        call("j4b_transpose", a.ptr, out.ptr, r, c, self.stream)
        return out

    # ---- conv2d (ComputeBackend.java:191-200) ----
    def _conv(self, entry, a, b, spec, out_shape, precision):
        out = self._new(out_shape)
        call(entry, a.ptr, b.ptr, out.ptr, a.shape[0], *spec.ints(), precision, self.stream)
        return out

    def conv2d(self, x: DeviceBuffer, w: DeviceBuffer, spec, precision: int = 0) -> DeviceBuffer:
        batch = spec.batch_of(x.shape, "conv2d input")
        if x.shape[1] != spec.input_size or tuple(w.shape) != spec.weight_shape():
            raise ValueError(f"conv2d shapes {x.shape} x {w.shape} do not match {spec}")
        return self._conv("j4b_conv2d", x, w, spec, spec.output_shape(batch), precision)

    def conv2d_grad_input(self, up: DeviceBuffer, w: DeviceBuffer, spec, precision: int = 0) -> DeviceBuffer:
        batch = spec.batch_of(up.shape, "conv2dGradInput upstream")
        if up.shape[1] != spec.output_size or tuple(w.shape) != spec.weight_shape():
            raise ValueError(f"conv2dGradInput shapes {up.shape} x {w.shape} do not match {spec}")
        return self._conv("j4b_conv2d_grad_input", up, w, spec, spec.input_shape(batch), precision)

    def conv2d_grad_weight(self, x: DeviceBuffer, up: DeviceBuffer, spec, precision: int = 0) -> DeviceBuffer:
        batch = spec.batch_of(x.shape, "conv2dGradWeight input")
        if x.shape[1] != spec.input_size or tuple(up.shape) != spec.output_shape(batch):
            raise ValueError(f"conv2dGradWeight shapes {x.shape} x {up.shape} do not match {spec}")
        return self._conv("j4b_conv2d_grad_weight", x, up, spec, spec.weight_shape(), precision)

    def matmul(self, a: DeviceBuffer, b: DeviceBuffer, precision: int = 0) -> DeviceBuffer:
        if len(a.shape) != 2 or len(b.shape) != 2 or a.shape[1] != b.shape[0]:
            raise ValueError(f"incompatible matmul shapes: {a.shape} x {b.shape}")
        m, k = a.shape
        n = b.shape[1]
        if min(m, k, n) < 1:
            raise ValueError("matmul dimensions must be positive")
        out = self._new((m, n))
        call("j4b_matmul", a.ptr, b.ptr, out.ptr, 1, m, k, n, precision, self.stream)
        return out

    def batched_matmul(self, a: DeviceBuffer, b: DeviceBuffer, precision: int = 0) -> DeviceBuffer:
        if (len(a.shape) != 3 or len(b.shape) != 3 or a.shape[0] != b.shape[0]
                or a.shape[2] != b.shape[1]):
            raise ValueError(f"incompatible batched matmul shapes: {a.shape} x {b.shape}")
        bt, m, k = a.shape
        n = b.shape[2]
        if min(bt, m, k, n) < 1:
            raise ValueError("matmul dimensions must be positive")
        out = self._new((bt, m, n))
        call("j4b_matmul", a.ptr, b.ptr, out.ptr, bt, m, k, n, precision, self.stream)
        return out

    def slice_axis0(self, a: DeviceBuffer, index: int) -> DeviceBuffer:
        if len(a.shape) < 1 or index < 0 or index >= a.shape[0]:
            raise ValueError(f"axis-0 index {index} is out of bounds for {a.shape}")
        size = a.size // a.shape[0]
        out = self._new(a.shape[1:])
        call("j4b_d2d", out.ptr, a.ptr + 4 * index * size, 4 * size, self.stream)
        return out

    def stack_axis0(self, inputs: list) -> DeviceBuffer:
        if not inputs:
            raise ValueError("stackAxis0 requires at least one input")
        first = inputs[0]
        for x in inputs:
            if x.shape != first.shape:
                raise ValueError("stackAxis0 inputs must have identical shape, dtype, and device")
        out = self._new((len(inputs),) + first.shape)
        for i, x in enumerate(inputs):
            call("j4b_d2d", out.ptr + 4 * i * first.size, x.ptr, 4 * first.size, self.stream)
        return out

    def reshape(self, a: DeviceBuffer, target) -> DeviceBuffer:
        if _prod(target) != a.size:
            raise ValueError(f"cannot reshape {a.shape} to {tuple(target)}")
        out = self._new(target)
        call("j4b_d2d", out.ptr, a.ptr, 4 * a.size, self.stream)
        return out

    def broadcast_to(self, a: DeviceBuffer, target) -> DeviceBuffer:
        target = tuple(int(d) for d in target)
        if a.shape == target:
            return a
        if broadcast_shape(a.shape, target) != target:
            raise ValueError(f"cannot broadcast shape {a.shape} to {target}")
        src = (ctypes.c_int64 * max(len(a.shape), 1))(*a.shape)
        dst = (ctypes.c_int64 * len(target))(*target)
        out = self._new(target)
        call("j4b_broadcast_to", a.ptr, src, len(a.shape), dst, len(target), out.ptr, self.stream)
        return out

    def _index_map(self, indices, bound: int) -> torch.Tensor:
        m = np.ascontiguousarray(np.asarray(indices, dtype=np.int32).reshape(-1))
        if m.size and (m.min() < -1 or m.max() >= bound):
            raise ValueError("index out of bounds")
        return torch.from_numpy(m).to(self._torch_device)

    def reindex(self, a: DeviceBuffer, target, indices) -> DeviceBuffer:
        if len(indices) != _prod(target):
            raise ValueError("index map size")
        m = self._index_map(indices, a.size)
        out = self._new(target)
        call("j4b_reindex", a.ptr, a.size, m.data_ptr(), out.size, out.ptr, self.stream)
        return out

    def scatter_add(self, a: DeviceBuffer, target, indices) -> DeviceBuffer:
        if len(indices) != a.size:
            raise ValueError("index map size")
        n = _prod(target)
        m = self._index_map(indices, n)
        out = self._new(target)
        call("j4b_scatter_add", a.ptr, a.size, m.data_ptr(), n, out.ptr, self.stream)
        return out

    # ---- reductions (ComputeBackend.java:150-177) ----
    def reduce_sum(self, a: DeviceBuffer) -> DeviceBuffer:
        out = self._new((1,))
        call("j4b_reduce_sum", a.ptr, a.size, out.ptr, self.stream)
        return out

    def reduce_max(self, a: DeviceBuffer) -> DeviceBuffer:
        out = self._new((1,))
        call("j4b_reduce_max", a.ptr, a.size, out.ptr, self.stream)
        return out

    @staticmethod
    def _axis(shape, axis: int):
        if axis < 0 or axis >= len(shape):
            raise ValueError(f"axis {axis} is out of bounds for shape {shape}")
        return _prod(shape[:axis]), shape[axis], _prod(shape[axis + 1:])

    @staticmethod
    def _reduced(shape, axis, keep):
        return tuple(1 if i == axis else d for i, d in enumerate(shape)) if keep else \
            tuple(d for i, d in enumerate(shape) if i != axis)

    def sum_axis0(self, a: DeviceBuffer) -> DeviceBuffer:
        if len(a.shape) != 2:
            raise ValueError(f"sumAxis0 requires a rank-2 tensor, got {a.shape}")
        return self.sum_axis(a, 0, False)

    def sum_axis(self, a: DeviceBuffer, axis: int, keep_dims: bool = False) -> DeviceBuffer:
        o, n, i = self._axis(a.shape, axis)
        out = self._new(self._reduced(a.shape, axis, keep_dims))
        call("j4b_sum_axis", a.ptr, o, n, i, out.ptr, self.stream)
        return out

    def max_axis(self, a: DeviceBuffer, axis: int, keep_dims: bool = False) -> DeviceBuffer:
        o, n, i = self._axis(a.shape, axis)
        out = self._new(self._reduced(a.shape, axis, keep_dims))
        call("j4b_max_axis", a.ptr, o, n, i, out.ptr, self.stream)
        return out

    def arg_max_axis(self, a: DeviceBuffer, axis: int) -> DeviceBuffer:
        o, n, i = self._axis(a.shape, axis)
        out = self._new(self._reduced(a.shape, axis, False))
        call("j4b_argmax_axis", a.ptr, o, n, i, out.ptr, self.stream)
        return out

    def max_axis_backward(self, upstream: DeviceBuffer, inp: DeviceBuffer, axis: int) -> DeviceBuffer:
        o, n, i = self._axis(inp.shape, axis)
        if upstream.size != o * i:
            raise ValueError(f"maxAxisBackward gradient shape {upstream.shape} is incompatible "
                             f"with input {inp.shape} and axis {axis}")
        out = self._new(inp.shape)
        call("j4b_max_axis_backward", upstream.ptr, inp.ptr, o, n, i, out.ptr, self.stream)
        return out

    # ---- lifecycle ----
    # ---- compiled tapes (ExecutionPlan.execute, ExecutionPlan.java:77-132) ----
    def execute_tape(self, tape, plan: dict, buffers: list) -> list:
        """Replays a recorded tape (jax4j_b200.jit.Tape) on the engine: compiled once per plan
        (j4b_tape_compile), launched per call (j4b_tape_launch) into fresh output buffers."""
        handle = plan.get("engine")
        if handle is None:
            handle = TapeHandle(self, tape)
            plan["engine"] = handle
        return handle.run(buffers)

    def sync(self) -> None:
        torch.cuda.current_stream(self._torch_device).synchronize()
        call("j4b_sync", self.device)

    def release(self, buf) -> None:
        """Idempotent (Tensor.close contract, core/tensor/Tensor.java:510-519)."""
        if isinstance(buf, DeviceBuffer) and not buf.released:
            buf.released = True
            buf.tensor = torch.empty(0, device=self._torch_device)

    # ---- QuantizedOps (QuantizedOps.java:19-34) ----
    def supported_quant_types(self) -> set:
        ids = (ctypes.c_int * 8)()
        n = ctypes.c_int(0)
        call("j4b_quant_supported", ids, 8, ctypes.byref(n))
        return {QUANT_NAMES[ids[i]] for i in range(n.value)}

    def upload_quantized(self, blocks, qtype: int, logical_shape) -> QuantBuffer:
        if len(logical_shape) != 2:
            raise ValueError("quantized matrices are rank 2")
        rows, cols = (int(d) for d in logical_shape)
        handle = ctypes.c_void_p()
        if isinstance(blocks, torch.Tensor):
            if not blocks.is_cuda or blocks.dtype != torch.uint8:
                raise ValueError("device blobs must be CUDA uint8 tensors")
            call("j4b_quant_upload_device", self.device, blocks.data_ptr(), blocks.numel(), qtype,
                 rows, cols, ctypes.byref(handle))
        else:
            arr = np.ascontiguousarray(np.asarray(blocks, dtype=np.uint8).reshape(-1))
            call("j4b_quant_upload", self.device, arr.ctypes.data_as(ctypes.c_void_p), arr.nbytes,
                 qtype, rows, cols, ctypes.byref(handle))
        return QuantBuffer(handle.value, qtype, (rows, cols))

    def quant_matvec(self, w: QuantBuffer, x: DeviceBuffer, add: DeviceBuffer | None = None,
                     out: DeviceBuffer | None = None):
        """y = W x (+ add). x of shape (cols,) is the reference call; (batch, cols) is batched.
        `out`, when given, is a preallocated buffer of batch * rows floats that receives y
        (a decode loop reuses it instead of allocating an output per call)."""
        rows, cols = w.shape
        if x.shape[-1] != cols or len(x.shape) > 2:
            raise ValueError(f"quantMatvec shape mismatch: {w.shape} x {x.shape}")
        batch = 1 if len(x.shape) == 1 else x.shape[0]
        out_shape = (rows,) if len(x.shape) == 1 else (batch, rows)
        if add is not None and add.size != batch * rows:
            raise ValueError(f"quantMatvecAdd addend shape {add.shape} does not match {out_shape}")
        if out is None:
            out = self._new(out_shape)
        elif out.size != batch * rows:
            raise ValueError(f"quantMatvec output holds {out.size} floats, the product needs {batch * rows}")
        call("j4b_quant_matvec", ctypes.c_void_p(w.handle), x.ptr, add.ptr if add else 0, out.ptr,
             batch, self.stream)
        return out

    def quant_matvec_host(self, w: QuantBuffer, x_host: torch.Tensor, y_host: torch.Tensor,
                          stream: int | None = None) -> None:
        """quantMatvec with host buffers (j4b_quant_matvec_host): x_host [batch, cols] and y_host
        [batch, rows] are contiguous f32 CPU tensors, pinned for asynchronous copies; y_host holds
        the product once the stream has been synchronised. `stream` defaults to PyTorch's current
        stream (a decode loop passes its handle once instead of looking it up every call)."""
        rows, cols = w.shape
        n = x_host.numel()
        if n % cols or not 1 <= n // cols <= 16 or y_host.numel() != n // cols * rows:
            raise ValueError(f"host quantMatvec shapes: W {w.shape}, x {tuple(x_host.shape)}, "
                             f"y {tuple(y_host.shape)} (batch 1..16)")
        call("j4b_quant_matvec_host", w.handle, x_host.data_ptr(), n // cols, y_host.data_ptr(),
             self.stream if stream is None else stream)

    def quant_matvec_host_plan(self, w: QuantBuffer, x_host: torch.Tensor, y_host: torch.Tensor) -> "QuantPlan":
        """quant_matvec_host recorded once (j4b_quant_matvec_host_plan): `plan.run(stream)` then
        replays the copy-in, the GEMV and the copy-out with one graph launch. The plan keeps x_host,
        y_host and w alive."""
        rows, cols = w.shape
        n = x_host.numel()
        if n % cols or not 1 <= n // cols <= 16 or y_host.numel() != n // cols * rows:
            raise ValueError(f"host quantMatvec shapes: W {w.shape}, x {tuple(x_host.shape)}, "
                             f"y {tuple(y_host.shape)} (batch 1..16)")
        return QuantPlan.make(w, x_host, y_host, n // cols, None, 0, self.stream)

    def quant_matvec_add(self, w: QuantBuffer, x: DeviceBuffer, add: DeviceBuffer):
        return self.quant_matvec(w, x, add)

    def quant_gemm(self, w: QuantBuffer, x: DeviceBuffer, precision: int = 1) -> DeviceBuffer:
        """Prefill projection y [m, rows] = x [m, cols] . W^T on the tensor cores (j4b_quant_gemm)."""
        rows, cols = w.shape
        if len(x.shape) != 2 or x.shape[1] != cols:
            raise ValueError(f"quant_gemm expects x [m, {cols}], got {x.shape}")
        out = self._new((x.shape[0], rows))
        call("j4b_quant_gemm", ctypes.c_void_p(w.handle), x.ptr, out.ptr, x.shape[0], precision,
             self.stream)
        return out

    def quant_gather_row(self, w: QuantBuffer, row: int) -> DeviceBuffer:
        if len(w.shape) != 2:
            raise ValueError(f"quantGatherRow requires a rank-2 quantized matrix, got {w.shape}")
        out = self._new((w.shape[1],))
        call("j4b_quant_gather_row", ctypes.c_void_p(w.handle), row, out.ptr, self.stream)
        return out

    def quantize(self, w: DeviceBuffer, qtype: int) -> torch.Tensor:
        """Encodes an f32 matrix on the device into GGUF blocks (a CUDA uint8 tensor)."""
        rows, cols = w.shape
        be, bb = QUANT_BLOCK[qtype]
        if cols % be:
            raise ValueError(f"{QUANT_NAMES[qtype]} tensor is not block-aligned: {cols} columns")
        out = torch.empty(rows * (cols // be) * bb, dtype=torch.uint8, device=self._torch_device)
        call("j4b_quantize", qtype, w.ptr, rows, cols, out.data_ptr(), self.stream)
        return out
