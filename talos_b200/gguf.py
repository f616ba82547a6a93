"""GGUF v3 container: reader and writer.

The reader mirrors Talos's ``GgufFile`` (Tsuskov/talos ``src/gguf/reader.rs:173-351``):
header, typed metadata, tensor index, 32-byte-aligned data section, zero-copy
tensor views, and the same errors (bad magic, version != 3, truncated index,
unsupported value or tensor types, data past the end of the file).

The writer produces the layout the reference's tests write by hand
(``tests/gqa.rs:24-108``, ``tests/forward_gpu.rs:25-144``): metadata, tensor infos
with 32-byte aligned offsets relative to the data section, padding, data.
"""
from __future__ import annotations

import mmap
import struct
from dataclasses import dataclass, field

import numpy as np

ALIGNMENT = 32

# Metadata value type tags (src/gguf/reader.rs:24-30).
T_UINT32, T_INT32, T_FLOAT32, T_BOOL, T_STRING, T_ARRAY = 4, 5, 6, 7, 8, 9

# ggml tensor types (src/gguf/dtype.rs:31-41).
F32, Q4_0, Q8_0, Q6_K = 0, 2, 8, 14
BLOCK_ELEMS = {F32: 1, Q4_0: 32, Q8_0: 32, Q6_K: 256}
BLOCK_BYTES = {F32: 4, Q4_0: 18, Q8_0: 34, Q6_K: 210}
TYPE_NAMES = {F32: "F32", Q4_0: "Q4_0", Q8_0: "Q8_0", Q6_K: "Q6_K"}


class GgufError(ValueError):
    pass


def raw_nbytes(gtype: int, n_elems: int) -> int:
    be = BLOCK_ELEMS[gtype]
    if n_elems % be:
        raise GgufError(f"{n_elems} elements is not a multiple of block {be}")
    return n_elems // be * BLOCK_BYTES[gtype]


@dataclass
class TensorInfo:
    """One tensor index entry (src/gguf/reader.rs:32-49). ``dims`` are in GGUF
    ``ne`` order: a row-major [rows, cols] matrix has dims [cols, rows]."""

    name: str
    dims: list[int]
    dtype: int
    offset: int

    def elem_count(self) -> int:
        n = 1
        for d in self.dims:
            n *= d
        return n


class _Cursor:
    """Bounds-checked reads (src/gguf/reader.rs:79-132)."""

    def __init__(self, buf):
        self.b = buf
        self.pos = 0

    def take(self, n: int):
        end = self.pos + n
        if n < 0 or end > len(self.b):
            raise GgufError(f"unexpected end of file (need {n} bytes at {self.pos})")
        s = self.b[self.pos:end]
        self.pos = end
        return s

    def u32(self):
        return struct.unpack("<I", self.take(4))[0]

    def i32(self):
        return struct.unpack("<i", self.take(4))[0]

    def u64(self):
        return struct.unpack("<Q", self.take(8))[0]

    def f32(self):
        return struct.unpack("<f", self.take(4))[0]

    def string(self):
        n = self.u64()
        raw = bytes(self.take(n))
        try:
            return raw.decode("utf-8")
        except UnicodeDecodeError as e:
            raise GgufError("metadata string is not valid UTF-8") from e


def _read_value(c: _Cursor, tag: int):
    """src/gguf/reader.rs:135-171"""
    if tag == T_UINT32:
        return ("u32", c.u32())
    if tag == T_FLOAT32:
        return ("f32", c.f32())
    if tag == T_BOOL:
        return ("bool", c.take(1)[0] != 0)
    if tag == T_STRING:
        return ("str", c.string())
    if tag == T_ARRAY:
        inner = c.u32()
        count = c.u64()
        if inner == T_STRING:
            if count > len(c.b):
                raise GgufError(f"unexpected end of file (array of {count})")
            return ("arr_str", [c.string() for _ in range(count)])
        if inner == T_INT32:
            raw = c.take(4 * count)
            return ("arr_i32", list(np.frombuffer(bytes(raw), "<i4").astype(int)))
        if inner == T_FLOAT32:
            raw = c.take(4 * count)
            return ("arr_f32", list(np.frombuffer(bytes(raw), "<f4").astype(float)))
        raise GgufError(f"unsupported array element type tag {inner}")
    raise GgufError(f"unsupported metadata value type tag {tag}")


class GgufFile:
    """A parsed GGUF file; tensor data stays in the (memory-mapped) buffer."""

    def __init__(self, buf, owner=None):
        self._buf = buf
        self._owner = owner
        self.meta: dict[str, tuple[str, object]] = {}
        self._tensors: list[TensorInfo] = []
        self._by_name: dict[str, int] = {}
        self.data_start = 0
        self._parse()

    @classmethod
    def open(cls, path: str) -> "GgufFile":
        f = open(path, "rb")
        try:
            mm = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
        except ValueError:  # empty file
            f.close()
            return cls(b"")
        f.close()
        return cls(memoryview(mm), owner=mm)

    @classmethod
    def from_bytes(cls, data: bytes) -> "GgufFile":
        return cls(memoryview(bytes(data)))

    def _parse(self):
        """src/gguf/reader.rs:193-246"""
        c = _Cursor(self._buf)
        magic = bytes(c.take(4))
        if magic != b"GGUF":
            raise GgufError(f"not a GGUF file (bad magic {magic!r})")
        version = c.u32()
        if version != 3:
            raise GgufError(f"unsupported GGUF version {version} (expected 3)")
        n_t = c.u64()
        n_kv = c.u64()
        for _ in range(n_kv):
            key = c.string()
            tag = c.u32()
            try:
                self.meta[key] = _read_value(c, tag)
            except GgufError as e:
                raise GgufError(f"reading metadata key {key!r}: {e}") from e
        for _ in range(n_t):
            name = c.string()
            nd = c.u32()
            dims = [c.u64() for _ in range(nd)]
            tag = c.u32()
            if tag not in BLOCK_ELEMS:
                raise GgufError(f"tensor {name!r} has unsupported ggml type {tag}")
            off = c.u64()
            self._by_name[name] = len(self._tensors)
            self._tensors.append(TensorInfo(name, dims, tag, off))
        ds = (c.pos + ALIGNMENT - 1) // ALIGNMENT * ALIGNMENT
        if ds > len(self._buf):
            raise GgufError(f"data section start {ds} past end of file {len(self._buf)}")
        self.data_start = ds

    # --- metadata (src/gguf/reader.rs:248-288)
    def metadata(self, key):
        v = self.meta.get(key)
        return None if v is None else v[1]

    def _get(self, key, kind):
        v = self.meta.get(key)
        return v[1] if v is not None and v[0] == kind else None

    def get_u32(self, key):
        return self._get(key, "u32")

    def get_f32(self, key):
        return self._get(key, "f32")

    def get_str(self, key):
        return self._get(key, "str")

    def get_bool(self, key):
        return self._get(key, "bool")

    def get_arr_str(self, key):
        return self._get(key, "arr_str")

    def get_arr_i32(self, key):
        return self._get(key, "arr_i32")

    def get_arr_f32(self, key):
        return self._get(key, "arr_f32")

    # --- tensors (src/gguf/reader.rs:290-351)
    def tensors(self) -> list[TensorInfo]:
        return self._tensors

    def tensor_info(self, name: str) -> TensorInfo | None:
        i = self._by_name.get(name)
        return None if i is None else self._tensors[i]

    def _range(self, info: TensorInfo, nbytes: int) -> memoryview:
        start = self.data_start + info.offset
        end = start + nbytes
        if end > len(self._buf):
            raise GgufError(f"tensor {info.name!r} data range past end of file")
        return self._buf[start:end]

    def tensor_f32(self, name: str) -> np.ndarray:
        info = self.tensor_info(name)
        if info is None:
            raise GgufError(f"no tensor named {name!r}")
        if info.dtype != F32:
            raise GgufError(f"tensor {name!r} is {TYPE_NAMES[info.dtype]}, not F32")
        mv = self._range(info, info.elem_count() * 4)
        return np.frombuffer(mv, dtype="<f4")

    def tensor_raw(self, name: str) -> tuple[memoryview, int]:
        info = self.tensor_info(name)
        if info is None:
            raise GgufError(f"no tensor named {name!r}")
        n = info.elem_count()
        be = BLOCK_ELEMS[info.dtype]
        if n % be:
            raise GgufError(f"tensor {name!r} has {n} elems, not a multiple of block {be}")
        return self._range(info, n // be * BLOCK_BYTES[info.dtype]), info.dtype


# ----------------------------------------------------------------- writer

def _put_str(out: bytearray, s: str):
    b = s.encode("utf-8")
    out += struct.pack("<Q", len(b))
    out += b


@dataclass
class _PendingTensor:
    name: str
    dims: list[int]
    dtype: int
    nbytes: int
    data: object = None  # bytes-like, or a callable returning bytes-like (streamed)


@dataclass
class GgufWriter:
    """Builds a GGUF v3 file. Tensors are given as raw bytes, or as a callable
    that returns them when the data section is written (so big models stream)."""

    kv: bytearray = field(default_factory=bytearray)
    n_kv: int = 0
    tensors: list = field(default_factory=list)

    def _key(self, k, tag):
        _put_str(self.kv, k)
        self.kv += struct.pack("<I", tag)
        self.n_kv += 1

    def add_u32(self, k, v):
        self._key(k, T_UINT32)
        self.kv += struct.pack("<I", v)

    def add_i32(self, k, v):
        self._key(k, T_INT32)
        self.kv += struct.pack("<i", v)

    def add_f32(self, k, v):
        self._key(k, T_FLOAT32)
        self.kv += struct.pack("<f", v)

    def add_bool(self, k, v):
        self._key(k, T_BOOL)
        self.kv += bytes([1 if v else 0])

    def add_str(self, k, v):
        self._key(k, T_STRING)
        _put_str(self.kv, v)

    def add_arr_str(self, k, vals):
        self._key(k, T_ARRAY)
        self.kv += struct.pack("<IQ", T_STRING, len(vals))
        for s in vals:
            _put_str(self.kv, s)

    def add_arr_i32(self, k, vals):
        self._key(k, T_ARRAY)
        self.kv += struct.pack("<IQ", T_INT32, len(vals))
        self.kv += np.asarray(vals, "<i4").tobytes()

    def add_arr_f32(self, k, vals):
        self._key(k, T_ARRAY)
        self.kv += struct.pack("<IQ", T_FLOAT32, len(vals))
        self.kv += np.asarray(vals, "<f4").tobytes()

    def add_tensor(self, name: str, dims: list[int], dtype: int, data):
        """``dims`` in GGUF ne order ([cols, rows] for a row-major matrix)."""
        n = 1
        for d in dims:
            n *= d
        nbytes = raw_nbytes(dtype, n)
        if not callable(data):
            data = bytes(data) if not isinstance(data, (bytes, bytearray, memoryview)) else data
            if len(data) != nbytes:
                raise GgufError(f"{name}: {len(data)} bytes, expected {nbytes}")
        self.tensors.append(_PendingTensor(name, list(dims), dtype, nbytes, data))

    def _header(self) -> tuple[bytearray, list[int]]:
        buf = bytearray(b"GGUF")
        buf += struct.pack("<IQQ", 3, len(self.tensors), self.n_kv)
        buf += self.kv
        offsets, off = [], 0
        for t in self.tensors:
            offsets.append(off)
            off = (off + t.nbytes + ALIGNMENT - 1) // ALIGNMENT * ALIGNMENT
        for t, o in zip(self.tensors, offsets):
            _put_str(buf, t.name)
            buf += struct.pack("<I", len(t.dims))
            for d in t.dims:
                buf += struct.pack("<Q", d)
            buf += struct.pack("<IQ", t.dtype, o)
        while len(buf) % ALIGNMENT:
            buf.append(0)
        return buf, offsets

    def _chunks(self):
        head, offsets = self._header()
        yield head
        pos = 0
        for t, o in zip(self.tensors, offsets):
            if o > pos:
                yield bytes(o - pos)
                pos = o
            data = t.data() if callable(t.data) else t.data
            if len(data) != t.nbytes:
                raise GgufError(f"{t.name}: produced {len(data)} bytes, expected {t.nbytes}")
            yield data
            pos += t.nbytes

    def to_bytes(self) -> bytes:
        return b"".join(bytes(c) for c in self._chunks())

    def write(self, path: str):
        with open(path, "wb") as f:
            for c in self._chunks():
                f.write(c)
