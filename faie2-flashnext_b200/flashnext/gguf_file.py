"""GGUF v3 files: a reader (memory-mapped tensors) and a writer, for the model loader (runner.py).

Layout of a GGUF v3 file (little-endian): the magic b"GGUF", uint32 version, uint64 tensor count, uint64 metadata
count; the metadata entries (string key, uint32 value type, value); the tensor infos (string name, uint32 number of
dimensions, uint64 dimensions innermost first, uint32 ggml type, uint64 offset into the data section); padding to the
alignment (metadata "general.alignment", default 32); the data section, each tensor at its offset (a multiple of the
alignment). A string is a uint64 byte length and UTF-8 bytes; an array value is a uint32 element type, a uint64 count
and the elements. The reference reads the same files with its own parser (gguf_open, engine/faie2fn.cu:197-260; the
general.alignment key at :239, the data start at :254); ggml type ids are the engine's format ids (fn_common.cuh).
"""

from __future__ import annotations

import os
import struct

import numpy as np

from synth import TYPES

MAGIC = b"GGUF"
ALIGN = 32
# metadata value types
U8, I8, U16, I16, U32, I32, F32, BOOL, STR, ARR, U64, I64, F64 = range(13)
_SCALAR = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<?", U64: "<Q",
           I64: "<q", F64: "<d"}
GGML_F32, GGML_F16 = 0, 1
# ggml type -> (values per block, bytes per block): the engine's formats and the float vectors
_BLOCK = {GGML_F32: (1, 4), GGML_F16: (1, 2), **{t: (qk, tb) for t, (_, qk, tb) in TYPES.items()}}


class GGUFError(ValueError):
    pass


class _Cursor:
    def __init__(self, buf, path):
        self.b, self.o, self.path = buf, 0, path

    def take(self, n):
        if self.o + n > len(self.b):
            raise GGUFError(f"{self.path}: truncated at byte {self.o}")
        v = self.b[self.o:self.o + n]
        self.o += n
        return v

    def scalar(self, t):
        fmt = _SCALAR[t]
        return struct.unpack(fmt, self.take(struct.calcsize(fmt)))[0]

    def string(self):
        n = self.scalar(U64)
        try:
            return bytes(self.take(n)).decode("utf-8")
        except UnicodeDecodeError as e:
            raise GGUFError(f"{self.path}: a string that is not UTF-8 at byte {self.o - n}") from e

    def value(self, t):
        if t == STR:
            return self.string()
        if t == ARR:
            et, n = self.scalar(U32), self.scalar(U64)
            if et not in _SCALAR and et not in (STR, ARR):
                raise GGUFError(f"{self.path}: bad array element type {et}")
            return [self.value(et) for _ in range(n)]
        if t not in _SCALAR:
            raise GGUFError(f"{self.path}: bad metadata value type {t}")
        return self.scalar(t)


class GGUFTensor:
    """One tensor: name, ggml type, dims (innermost first), and its bytes (a read-only view of the mapped file)."""

    def __init__(self, name, qtype, dims, data):
        self.name, self.qtype, self.dims, self.data = name, qtype, tuple(dims), data

    @property
    def cols(self) -> int:
        return self.dims[0]

    @property
    def rows(self) -> int:
        return int(np.prod(self.dims[1:], dtype=np.int64)) if len(self.dims) > 1 else 1

    def rows_u8(self) -> np.ndarray:
        """The tensor as GGUF rows, uint8 [rows, row_bytes]."""
        return self.data.reshape(self.rows, -1)

    def f32(self) -> np.ndarray:
        """An F32 / F16 tensor as float32, shape (rows, cols) or (cols,) for one row."""
        if self.qtype == GGML_F32:
            a = self.data.view(np.float32)
        elif self.qtype == GGML_F16:
            a = self.data.view(np.float16).astype(np.float32)
        else:
            raise GGUFError(f"{self.name}: expected F32 or F16, got ggml type {self.qtype}")
        return a.reshape(self.rows, self.cols) if len(self.dims) > 1 else a.reshape(self.cols)


def _nbytes(qtype: int, dims) -> int:
    if qtype not in _BLOCK:
        raise GGUFError(f"unsupported ggml type {qtype}")
    qk, tb = _BLOCK[qtype]
    rows = int(np.prod(dims[1:], dtype=np.int64)) if len(dims) > 1 else 1
    if dims[0] % qk:
        raise GGUFError(f"row length {dims[0]} is not a multiple of the block size of ggml type {qtype}")
    return rows * (dims[0] // qk) * tb


def read(path: str):
    """-> (metadata dict, {name: GGUFTensor}); tensor bytes are views of a read-only memory map of the file."""
    if os.path.getsize(path) < 24:  # magic, version and the two counts (and numpy maps no empty file)
        raise GGUFError(f"{path}: truncated at byte 0")
    buf = np.memmap(path, dtype=np.uint8, mode="r")
    c = _Cursor(buf, path)
    if bytes(c.take(4)) != MAGIC:
        raise GGUFError(f"{path}: not a GGUF file")
    ver = c.scalar(U32)
    if ver not in (2, 3):
        raise GGUFError(f"{path}: GGUF version {ver} not supported")
    n_t, n_kv = c.scalar(U64), c.scalar(U64)
    meta = {}
    for _ in range(n_kv):
        k = c.string()
        meta[k] = c.value(c.scalar(U32))
    infos = []
    for _ in range(n_t):
        name = c.string()
        nd = c.scalar(U32)
        if not 1 <= nd <= 4:
            raise GGUFError(f"{path}: {name}: {nd} dimensions")
        dims = [c.scalar(U64) for _ in range(nd)]
        infos.append((name, dims, c.scalar(U32), c.scalar(U64)))
    align = int(meta.get("general.alignment", ALIGN))
    if align <= 0 or align & (align - 1):
        raise GGUFError(f"{path}: bad alignment {align}")
    base = (c.o + align - 1) // align * align
    tensors = {}
    for name, dims, qt, off in infos:
        n = _nbytes(qt, dims)
        if off % align or base + off + n > len(buf):
            raise GGUFError(f"{path}: {name}: data out of range")
        if name in tensors:
            raise GGUFError(f"{path}: duplicate tensor {name}")
        tensors[name] = GGUFTensor(name, qt, dims, buf[base + off:base + off + n])
    return meta, tensors


def _meta_type(v):
    if isinstance(v, bool):
        return BOOL
    if isinstance(v, int):
        return U32 if 0 <= v < 2**32 else I64
    if isinstance(v, float):
        return F32
    if isinstance(v, str):
        return STR
    if isinstance(v, (list, tuple)):
        return ARR
    raise TypeError(f"metadata value {v!r}")


def _put_value(out, t, v):
    if t == STR:
        b = v.encode("utf-8")
        out += struct.pack("<Q", len(b)) + b
    elif t == ARR:
        et = _meta_type(v[0]) if len(v) else U32
        out += struct.pack("<IQ", et, len(v))
        for e in v:
            _put_value(out, et, e)
    else:
        out += struct.pack(_SCALAR[t], v)


def write(path: str, meta: dict, tensors, data=None) -> None:
    """Write a GGUF v3 file. tensors: iterable of (name, ggml type, dims innermost first, bytes-like data); or, with
    `data` given, of (name, ggml type, dims) and `data` an iterable of the tensors' bytes in the same order, consumed
    once while the file is written (the header needs only the names, types and dims, so a model larger than host
    memory can be written tensor by tensor)."""
    tensors = list(tensors)
    if data is None:
        data = (t[3] for t in tensors)
    head = bytearray(MAGIC + struct.pack("<IQQ", 3, len(tensors), len(meta)))
    for k, v in meta.items():
        t = _meta_type(v)
        _put_value(head, STR, k)
        head += struct.pack("<I", t)
        _put_value(head, t, v)
    off, offs = 0, []
    for name, qt, dims, *_ in tensors:
        _put_value(head, STR, name)
        head += struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        head += struct.pack("<IQ", qt, off)
        offs.append(off)
        off = (off + _nbytes(qt, dims) + ALIGN - 1) // ALIGN * ALIGN
    with open(path, "wb") as f:
        f.write(head)
        f.write(b"\0" * ((-len(head)) % ALIGN))
        pos, it = 0, iter(data)
        for (name, qt, dims, *_), o in zip(tensors, offs):
            try:
                d = memoryview(np.ascontiguousarray(next(it))).cast("B")
            except StopIteration:
                raise GGUFError(f"{name}: no data") from None
            if len(d) != _nbytes(qt, dims):
                raise GGUFError(f"{name}: {len(d)} bytes for dims {dims} of ggml type {qt}")
            f.write(b"\0" * (o - pos))
            f.write(d)
            pos = o + len(d)
        if next(it, None) is not None:
            raise GGUFError("more data than tensors")
