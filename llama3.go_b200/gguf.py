"""GGUF v3 container: a minimal writer (synthetic models) and reader.

The reader follows the reference parser internal/gguf/gguf.go:
  * header, KV section and tensor infos, gguf.go:64-152;
  * value types 0..12, gguf.go:25-39 and readValue gguf.go:262-380;
  * data offset = end of tensor infos rounded up to ``general.alignment``
    (default 32, only honoured when stored as UINT32), gguf.go:154-234;
  * typed getters: ``get_u32`` accepts UINT32 and UINT64 <= 2**32-1 only,
    ``get_f32`` FLOAT32 only (gguf.go:391-432), which is why the synthetic
    writer stores counts as UINT32 and eps / rope base as FLOAT32.
"""
from __future__ import annotations

import os
import struct
from dataclasses import dataclass, field

import numpy as np

GGUF_MAGIC = b"GGUF"

# gguf.go:25-39
T_UINT8, T_INT8, T_UINT16, T_INT16, T_UINT32, T_INT32, T_FLOAT32, T_BOOL, \
    T_STRING, T_ARRAY, T_UINT64, T_INT64, T_FLOAT64 = range(13)

# q8_0.go:7-11
GGML_F32, GGML_F16, GGML_Q8_0 = 0, 1, 8

_SCALAR_FMT = {
    T_UINT8: "<B", T_INT8: "<b", T_UINT16: "<H", T_INT16: "<h",
    T_UINT32: "<I", T_INT32: "<i", T_FLOAT32: "<f", T_UINT64: "<Q",
    T_INT64: "<q", T_FLOAT64: "<d",
}
_NP_DTYPE = {
    T_UINT8: np.uint8, T_INT8: np.int8, T_UINT16: np.uint16,
    T_INT16: np.int16, T_UINT32: np.uint32, T_INT32: np.int32,
    T_FLOAT32: np.float32, T_UINT64: np.uint64, T_INT64: np.int64,
    T_FLOAT64: np.float64,
}


def tensor_nbytes(ggml_type: int, dims) -> int:
    """Byte size of a tensor; the reference never computes it (reader.go:31-37
    slices to end of file), so loaders derive it from type and dims."""
    n = 1
    for d in dims:
        n *= int(d)
    if ggml_type == GGML_F32:
        return 4 * n
    if ggml_type == GGML_F16:
        return 2 * n
    if ggml_type == GGML_Q8_0:
        if int(dims[0]) % 32:
            raise ValueError("Q8_0 tensor ne0 not a multiple of 32")
        return n // 32 * 34
    raise ValueError(f"unsupported ggml type {ggml_type}")


@dataclass
class TensorInfo:
    name: str
    dims: list            # ne0 first: [cols, rows] for matrices
    ggml_type: int
    offset: int           # relative to the data section


@dataclass
class GGUFFile:
    version: int
    kv: dict = field(default_factory=dict)      # key -> (type, value)
    tensors: list = field(default_factory=list)
    data_offset: int = 0
    alignment: int = 32
    _buf: object = None

    # typed getters, gguf.go:382-441
    def get_u32(self, key):
        t = self.kv.get(key)
        if t is None:
            return None
        typ, v = t
        if typ == T_UINT32:
            return int(v)
        if typ == T_UINT64 and v <= 0xFFFFFFFF:
            return int(v)
        return None

    def get_f32(self, key):
        t = self.kv.get(key)
        if t is None or t[0] != T_FLOAT32:
            return None
        return float(t[1])

    def get_string(self, key):
        t = self.kv.get(key)
        if t is None or t[0] != T_STRING:
            return None
        return t[1]

    def tensor(self, name):
        for ti in self.tensors:
            if ti.name == name:
                return ti
        return None

    def tensor_data(self, ti: TensorInfo) -> np.ndarray:
        start = self.data_offset + ti.offset
        n = tensor_nbytes(ti.ggml_type, ti.dims)
        return np.frombuffer(self._buf, dtype=np.uint8, count=n, offset=start)


class _Reader:
    def __init__(self, buf):
        self.buf = buf
        self.pos = 0

    def take(self, n):
        if self.pos + n > len(self.buf):
            raise EOFError("truncated gguf")
        b = self.buf[self.pos:self.pos + n]
        self.pos += n
        return b

    def scalar(self, typ):
        fmt = _SCALAR_FMT[typ]
        return struct.unpack(fmt, self.take(struct.calcsize(fmt)))[0]

    def string(self):
        n = self.scalar(T_UINT64)
        if n > 1 << 30:
            raise ValueError(f"string too large: {n}")
        return bytes(self.take(n)).decode("utf-8", errors="replace")

    def value(self, typ):
        if typ in _SCALAR_FMT:
            return self.scalar(typ)
        if typ == T_BOOL:
            return self.scalar(T_UINT8) != 0
        if typ == T_STRING:
            return self.string()
        if typ == T_ARRAY:
            et = self.scalar(T_UINT32)
            n = self.scalar(T_UINT64)
            if n > 1 << 28:
                raise ValueError(f"array too large: {n}")
            if et in _NP_DTYPE:
                dt = np.dtype(_NP_DTYPE[et])
                return np.frombuffer(bytes(self.take(n * dt.itemsize)), dtype=dt)
            return [self.value(et) for _ in range(n)]
        raise ValueError(f"unsupported gguf value type: {typ}")


def read_gguf(path_or_buf) -> GGUFFile:
    """Parse a GGUF file (path, bytes or a numpy memmap)."""
    if isinstance(path_or_buf, (str, os.PathLike)):
        buf = np.memmap(path_or_buf, dtype=np.uint8, mode="r")
    else:
        buf = path_or_buf
    mv = memoryview(buf) if not isinstance(buf, np.ndarray) else memoryview(buf).cast("B")
    r = _Reader(mv)
    if bytes(r.take(4)) != GGUF_MAGIC:
        raise ValueError("not a gguf file")
    version = r.scalar(T_UINT32)
    n_tensors = r.scalar(T_UINT64)
    n_kv = r.scalar(T_UINT64)
    f = GGUFFile(version=version)
    alignment = 32
    for _ in range(n_kv):
        key = r.string()
        typ = r.scalar(T_UINT32)
        val = r.value(typ)
        f.kv[key] = (typ, val)
        if key == "general.alignment" and typ == T_UINT32:
            alignment = int(val)
    for _ in range(n_tensors):
        name = r.string()
        nd = r.scalar(T_UINT32)
        dims = [r.scalar(T_UINT64) for _ in range(nd)]
        typ = r.scalar(T_UINT32)
        off = r.scalar(T_UINT64)
        f.tensors.append(TensorInfo(name, dims, typ, off))
    pos = r.pos
    if alignment > 0 and pos % alignment:
        pos += alignment - pos % alignment
    f.data_offset = pos
    f.alignment = alignment
    f._buf = buf
    return f


class GGUFWriter:
    """Writes GGUF v3: KV pairs, tensor infos, aligned tensor data."""

    def __init__(self, alignment=32):
        self.alignment = alignment
        self.kv = []          # (key, type, value[, elem_type])
        self.tensors = []     # (name, dims, ggml_type, array)
        self.add("general.alignment", T_UINT32, alignment)

    def add(self, key, typ, value, elem_type=None):
        self.kv.append((key, typ, value, elem_type))

    def add_tensor(self, name, dims, ggml_type, data: np.ndarray):
        want = tensor_nbytes(ggml_type, dims)
        if data.nbytes != want:
            raise ValueError(f"{name}: {data.nbytes} bytes, want {want}")
        self.tensors.append((name, list(dims), ggml_type, data))

    @staticmethod
    def _string(s):
        b = s.encode("utf-8")
        return struct.pack("<Q", len(b)) + b

    def _value(self, typ, v, elem_type=None):
        if typ in _SCALAR_FMT:
            return struct.pack(_SCALAR_FMT[typ], v)
        if typ == T_BOOL:
            return struct.pack("<B", 1 if v else 0)
        if typ == T_STRING:
            return self._string(v)
        if typ == T_ARRAY:
            out = struct.pack("<IQ", elem_type, len(v))
            if elem_type == T_STRING:
                return out + b"".join(self._string(s) for s in v)
            return out + np.asarray(v, dtype=_NP_DTYPE[elem_type]).tobytes()
        raise ValueError(typ)

    def write(self, path):
        head = bytearray()
        head += GGUF_MAGIC + struct.pack("<IQQ", 3, len(self.tensors), len(self.kv))
        for key, typ, v, et in self.kv:
            head += self._string(key) + struct.pack("<I", typ) + self._value(typ, v, et)
        off = 0
        offsets = []
        for name, dims, typ, data in self.tensors:
            if off % self.alignment:
                off += self.alignment - off % self.alignment
            offsets.append(off)
            off += data.nbytes
        for (name, dims, typ, data), o in zip(self.tensors, offsets):
            head += self._string(name) + struct.pack("<I", len(dims))
            head += b"".join(struct.pack("<Q", int(d)) for d in dims)
            head += struct.pack("<IQ", typ, o)
        pad = (-len(head)) % self.alignment
        head += b"\0" * pad
        with open(path, "wb") as fh:
            fh.write(head)
            pos = 0
            for (name, dims, typ, data), o in zip(self.tensors, offsets):
                if o > pos:
                    fh.write(b"\0" * (o - pos))
                    pos = o
                fh.write(memoryview(np.ascontiguousarray(data)).cast("B"))
                pos += data.nbytes
