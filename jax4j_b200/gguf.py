"""GGUF files: read the metadata and tensor directory of a GGUF (version 2 or 3) file, map its
tensor data, and upload its quantised matrices to the engine (QuantizedOps.uploadQuantized,
core/tensor/spi/QuantizedOps.java:23-24; type ids and block geometry as QuantType.java:4-13).

Layout (little-endian): magic "GGUF", uint32 version, uint64 tensor count, uint64 metadata
count; metadata entries (string key, uint32 value type, value); tensor infos (string name,
uint32 n_dims, uint64 dims[n_dims] with dims[0] the fastest-varying axis, uint32 type id, uint64
offset relative to the data section); the data section starts at the first multiple of
`general.alignment` (default 32) after the infos, and every tensor offset is a multiple of it.
Strings are a uint64 byte length followed by UTF-8 bytes. A rank-2 tensor with dims [ne0, ne1]
is a row-major matrix of ne1 rows and ne0 columns.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field

import numpy as np

MAGIC = b"GGUF"
DEFAULT_ALIGNMENT = 32

# metadata value types
UINT8, INT8, UINT16, INT16, UINT32, INT32, FLOAT32, BOOL, STRING, ARRAY, UINT64, INT64, FLOAT64 = range(13)
_SCALAR = {UINT8: "<B", INT8: "<b", UINT16: "<H", INT16: "<h", UINT32: "<I", INT32: "<i",
           FLOAT32: "<f", BOOL: "<?", UINT64: "<Q", INT64: "<q", FLOAT64: "<d"}

# ggml type id -> (name, block elements, block bytes); QuantType.java:4-13
TYPES = {0: ("F32", 1, 4), 1: ("F16", 1, 2), 2: ("Q4_0", 32, 18), 8: ("Q8_0", 32, 34),
         12: ("Q4_K", 256, 144), 14: ("Q6_K", 256, 210), 30: ("BF16", 1, 2),
         41: ("Q1_0", 256, 34), 42: ("Q2_0", 128, 34)}


def byte_size(type_id: int, elements: int) -> int:
    """QuantType.byteSizeFor (QuantType.java:46-53)."""
    if type_id not in TYPES:
        raise ValueError(f"unknown ggml quant type id: {type_id}")
    name, be, bb = TYPES[type_id]
    if elements % be:
        raise ValueError(f"{name} tensor is not block-aligned: {elements} elements, block={be}")
    return elements // be * bb


@dataclass
class TensorInfo:
    name: str
    dims: tuple        # GGUF order: dims[0] fastest
    type_id: int
    offset: int        # relative to the data section
    nbytes: int

    @property
    def shape(self) -> tuple:
        """Row-major logical shape (slowest axis first)."""
        return tuple(reversed(self.dims))


@dataclass
class GGUFFile:
    path: str
    version: int
    metadata: dict
    tensors: list
    data_offset: int
    alignment: int
    _map: np.memmap = field(default=None, repr=False)

    def tensor(self, name: str) -> TensorInfo:
        for t in self.tensors:
            if t.name == name:
                return t
        raise KeyError(f"no tensor named {name!r} in {self.path}")

    def data(self, name: str) -> np.ndarray:
        """The tensor's raw bytes (a read-only view of the mapped file)."""
        t = self.tensor(name)
        if self._map is None:
            self._map = np.memmap(self.path, dtype=np.uint8, mode="r")
        start = self.data_offset + t.offset
        return self._map[start:start + t.nbytes]


class _Reader:
    def __init__(self, buf: bytes):
        self.buf, self.pos = buf, 0

    def take(self, n: int) -> bytes:
        if self.pos + n > len(self.buf):
            raise ValueError("GGUF file is truncated")
        b = self.buf[self.pos:self.pos + n]
        self.pos += n
        return b

    def scalar(self, fmt: str):
        return struct.unpack(fmt, self.take(struct.calcsize(fmt)))[0]

    def string(self) -> str:
        return self.take(self.scalar("<Q")).decode("utf-8")

    def value(self, vtype: int):
        if vtype in _SCALAR:
            return self.scalar(_SCALAR[vtype])
        if vtype == STRING:
            return self.string()
        if vtype == ARRAY:
            etype, count = self.scalar("<I"), self.scalar("<Q")
            return [self.value(etype) for _ in range(count)]
        raise ValueError(f"unknown GGUF metadata value type {vtype}")


def read(path: str) -> GGUFFile:
    """Parses the header, metadata and tensor directory; tensor data stays on disk (memory-mapped
    on first access)."""
    with open(path, "rb") as f:
        head = f.read(24)
        if len(head) < 24 or head[:4] != MAGIC:
            raise ValueError(f"{path} is not a GGUF file")
        version, n_tensors, n_kv = struct.unpack("<IQQ", head[4:24])
        if version not in (2, 3):
            raise ValueError(f"unsupported GGUF version {version}")
        # the directory is small; read until it parses (grow the window if needed)
        size = 1 << 20
        while True:
            f.seek(0)
            buf = f.read(size)
            try:
                r = _Reader(buf)
                r.pos = 24
                meta = {}
                for _ in range(n_kv):
                    key = r.string()
                    meta[key] = r.value(r.scalar("<I"))
                infos = []
                for _ in range(n_tensors):
                    name = r.string()
                    nd = r.scalar("<I")
                    dims = tuple(r.scalar("<Q") for _ in range(nd))
                    tid = r.scalar("<I")
                    off = r.scalar("<Q")
                    n = int(np.prod(dims)) if dims else 1
                    infos.append(TensorInfo(name, dims, tid, off, byte_size(tid, n)))
                break
            except ValueError as e:
                if "truncated" in str(e) and len(buf) == size:
                    size *= 4
                    continue
                raise
    align = int(meta.get("general.alignment", DEFAULT_ALIGNMENT))
    if align <= 0 or align & (align - 1):
        raise ValueError(f"general.alignment must be a power of two, got {align}")
    data_offset = (r.pos + align - 1) // align * align
    for t in infos:
        if t.offset % align:
            raise ValueError(f"tensor {t.name} offset {t.offset} is not {align}-aligned")
    return GGUFFile(path, version, meta, infos, data_offset, align)


def _value_type(v) -> int:
    if isinstance(v, bool):
        return BOOL
    if isinstance(v, int):
        return INT64 if v < 0 else UINT64 if v >= 2 ** 32 else UINT32
    if isinstance(v, float):
        return FLOAT32
    if isinstance(v, str):
        return STRING
    if isinstance(v, (list, tuple)):
        return ARRAY
    raise TypeError(f"no GGUF metadata type for {type(v).__name__}")


def _pack_value(vtype: int, v) -> bytes:
    if vtype in _SCALAR:
        return struct.pack(_SCALAR[vtype], v)
    if vtype == STRING:
        b = v.encode("utf-8")
        return struct.pack("<Q", len(b)) + b
    et = _value_type(v[0]) if v else UINT32
    return struct.pack("<IQ", et, len(v)) + b"".join(_pack_value(et, x) for x in v)


def write(path: str, metadata: dict, tensors: list, alignment: int = DEFAULT_ALIGNMENT) -> None:
    """Writes a version-3 GGUF file. tensors: (name, shape (row-major), ggml type id, raw bytes)."""
    meta = dict(metadata)
    if alignment != DEFAULT_ALIGNMENT:
        meta["general.alignment"] = alignment
    out = bytearray(MAGIC + struct.pack("<IQQ", 3, len(tensors), len(meta)))
    for k, v in meta.items():
        vt = _value_type(v)
        out += _pack_value(STRING, k) + struct.pack("<I", vt) + _pack_value(vt, v)
    off, blobs = 0, []
    for name, shape, tid, raw in tensors:
        raw = np.ascontiguousarray(np.asarray(raw, dtype=np.uint8).reshape(-1)).tobytes()
        if len(raw) != byte_size(tid, int(np.prod(shape))):
            raise ValueError(f"tensor {name}: {len(raw)} bytes for shape {shape} of type {tid}")
        dims = tuple(reversed(shape))
        out += _pack_value(STRING, name) + struct.pack("<I", len(dims))
        out += b"".join(struct.pack("<Q", d) for d in dims) + struct.pack("<IQ", tid, off)
        blobs.append((off, raw))
        off = (off + len(raw) + alignment - 1) // alignment * alignment
    out += b"\0" * ((-len(out)) % alignment)
    base = len(out)
    out += b"\0" * off
    for o, raw in blobs:
        out[base + o:base + o + len(raw)] = raw
    with open(path, "wb") as f:
        f.write(out)


def load_quantized(backend, gguf: GGUFFile, names=None) -> dict:
    """Uploads the file's rank-2 block-quantised matrices (types the engine supports) as
    QuantBuffers keyed by tensor name. F32 and F16 tensors come back as f32 DeviceBuffers."""
    from ._lib import QUANT_BLOCK
    out = {}
    for t in gguf.tensors:
        if names is not None and t.name not in names:
            continue
        raw = np.asarray(gguf.data(t.name))
        if t.type_id in (0, 1):
            arr = raw.view(np.float32 if t.type_id == 0 else np.float16).astype(np.float32)
            out[t.name] = backend.upload(arr, t.shape)
        elif t.type_id in QUANT_BLOCK and len(t.dims) == 2:
            out[t.name] = backend.upload_quantized(raw, t.type_id, t.shape)
        elif names is not None:
            raise NotImplementedError(f"tensor {t.name}: type {TYPES.get(t.type_id, (t.type_id,))[0]} "
                                      f"of rank {len(t.dims)} is not supported by the engine")
    return out
