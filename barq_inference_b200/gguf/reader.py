"""Zero-copy GGUF reader.

Behavioural parity with the reference's ``GgufReader`` (``barq_core/src/gguf.rs:250-372``:
magic, version <= 3 header, the 13 metadata value types including nested arrays, tensor
infos, aligned data offset).  Unlike the reference, tensors are *not* dequantized at load
(``gguf.rs:415-519``): the file is memory-mapped and every tensor is exposed as a packed
``uint8`` view of its GGUF blocks, which is what the device kernels consume.
"""
from __future__ import annotations

import mmap
import os
import re
import struct
from dataclasses import dataclass, field
from typing import Any

import numpy as np

from .constants import (
    GGUF_DEFAULT_ALIGNMENT,
    GGUF_MAGIC,
    TYPE_TRAITS,
    GGMLType,
    GGUFValueType,
    row_nbytes,
)

_SCALAR_FMT = {
    GGUFValueType.UINT8: "<B",
    GGUFValueType.INT8: "<b",
    GGUFValueType.UINT16: "<H",
    GGUFValueType.INT16: "<h",
    GGUFValueType.UINT32: "<I",
    GGUFValueType.INT32: "<i",
    GGUFValueType.FLOAT32: "<f",
    GGUFValueType.BOOL: "<?",
    GGUFValueType.UINT64: "<Q",
    GGUFValueType.INT64: "<q",
    GGUFValueType.FLOAT64: "<d",
}

_NP_DTYPE = {
    GGUFValueType.UINT8: np.uint8,
    GGUFValueType.INT8: np.int8,
    GGUFValueType.UINT16: np.uint16,
    GGUFValueType.INT16: np.int16,
    GGUFValueType.UINT32: np.uint32,
    GGUFValueType.INT32: np.int32,
    GGUFValueType.FLOAT32: np.float32,
    GGUFValueType.BOOL: np.bool_,
    GGUFValueType.UINT64: np.uint64,
    GGUFValueType.INT64: np.int64,
    GGUFValueType.FLOAT64: np.float64,
}


class GGUFError(ValueError):
    pass


@dataclass
class TensorInfo:
    name: str
    shape: tuple[int, ...]  # ggml order: ne0 (innermost) first
    ggml_type: GGMLType
    offset: int  # relative to the data section
    data: np.ndarray | None = None  # packed uint8 view

    @property
    def n_elements(self) -> int:
        n = 1
        for d in self.shape:
            n *= d
        return n

    @property
    def nbytes(self) -> int:
        return self.n_elements // self.shape[0] * row_nbytes(self.ggml_type, self.shape[0])

    @property
    def torch_shape(self) -> tuple[int, ...]:
        """Row-major shape (outermost first), e.g. ``(n_out, n_in)`` for a weight."""
        return tuple(reversed(self.shape))

    def rows(self) -> np.ndarray:
        """Packed bytes as ``[n_rows, row_bytes]`` where a row is ``ne0`` elements."""
        return self.data.reshape(-1, row_nbytes(self.ggml_type, self.shape[0]))


@dataclass
class GGUFFile:
    path: str
    version: int
    metadata: dict[str, Any]
    metadata_types: dict[str, GGUFValueType]
    tensors: dict[str, TensorInfo]
    alignment: int
    data_offset: int
    _mm: Any = field(default=None, repr=False)

    def get(self, key: str, default: Any = None) -> Any:
        return self.metadata.get(key, default)

    @property
    def architecture(self) -> str:
        return str(self.metadata.get("general.architecture", "llama"))

    def tensor(self, name: str) -> TensorInfo:
        if name not in self.tensors:
            raise KeyError(f"tensor {name!r} not in {self.path}")
        return self.tensors[name]

    def close(self) -> None:
        for t in self.tensors.values():
            t.data = None
        if self._mm is not None and not hasattr(self._mm, "close"):  # native map: freed with its views
            self._mm = None
        if self._mm is not None:
            try:
                self._mm.close()
            except BufferError:
                pass  # views still alive; the map is released with them
            self._mm = None


class _Cursor:
    __slots__ = ("buf", "pos")

    def __init__(self, buf, pos: int = 0):
        self.buf = buf
        self.pos = pos

    def need(self, n: int) -> None:
        if self.pos + n > len(self.buf):
            raise GGUFError(f"truncated GGUF at byte {self.pos} (need {n} more)")

    def scalar(self, vt: GGUFValueType):
        fmt = _SCALAR_FMT[vt]
        n = struct.calcsize(fmt)
        self.need(n)
        (v,) = struct.unpack_from(fmt, self.buf, self.pos)
        self.pos += n
        return v

    def u32(self) -> int:
        return self.scalar(GGUFValueType.UINT32)

    def u64(self) -> int:
        return self.scalar(GGUFValueType.UINT64)

    def string(self) -> str:
        n = self.u64()
        if n > (1 << 32):
            raise GGUFError(f"implausible string length {n}")
        self.need(n)
        s = bytes(self.buf[self.pos : self.pos + n]).decode("utf-8", errors="replace")
        self.pos += n
        return s

    def value(self, vt: GGUFValueType, depth: int = 0):
        if vt == GGUFValueType.STRING:
            return self.string()
        if vt == GGUFValueType.ARRAY:
            if depth > 8:
                raise GGUFError("array nesting too deep")
            et = GGUFValueType(self.u32())
            n = self.u64()
            if et in _NP_DTYPE:
                dt = np.dtype(_NP_DTYPE[et]).newbyteorder("<")
                nb = n * dt.itemsize
                self.need(nb)
                arr = np.frombuffer(self.buf, dtype=dt, count=n, offset=self.pos).copy()
                self.pos += nb
                return arr.tolist() if n <= 64 else arr
            return [self.value(et, depth + 1) for _ in range(n)]
        return self.scalar(vt)


def _parse(buf, path: str) -> GGUFFile:
    c = _Cursor(buf)
    magic = c.u32()
    if magic != GGUF_MAGIC:
        raise GGUFError(f"{path}: bad magic 0x{magic:08x}")
    version = c.u32()
    if version < 1 or version > 3:
        raise GGUFError(f"{path}: unsupported GGUF version {version}")
    if version == 1:
        raise GGUFError("GGUF v1 (32-bit counts) is not supported")
    n_tensors = c.u64()
    n_kv = c.u64()
    if n_tensors > 10_000_000 or n_kv > 10_000_000:
        raise GGUFError("implausible tensor/kv count")
    md: dict[str, Any] = {}
    mdt: dict[str, GGUFValueType] = {}
    for _ in range(n_kv):
        key = c.string()
        vt = GGUFValueType(c.u32())
        md[key] = c.value(vt)
        mdt[key] = vt
    infos: dict[str, TensorInfo] = {}
    for _ in range(n_tensors):
        name = c.string()
        nd = c.u32()
        if nd > 8:
            raise GGUFError(f"tensor {name}: {nd} dims")
        shape = tuple(c.u64() for _ in range(nd))
        tt = GGMLType(c.u32())
        off = c.u64()
        infos[name] = TensorInfo(name, shape, tt, off)
    alignment = int(md.get("general.alignment", GGUF_DEFAULT_ALIGNMENT))
    data_offset = (c.pos + alignment - 1) // alignment * alignment
    for t in infos.values():
        if t.ggml_type not in TYPE_TRAITS:
            raise GGUFError(f"tensor {t.name}: unsupported ggml type {t.ggml_type.name}")
        start = data_offset + t.offset
        if start + t.nbytes > len(buf):
            raise GGUFError(f"tensor {t.name} extends past end of file")
        t.data = np.frombuffer(buf, dtype=np.uint8, count=t.nbytes, offset=start)
    return GGUFFile(path, version, md, mdt, infos, alignment, data_offset)


def _native():
    if os.environ.get("BARQ_GGUF_NATIVE", "1") == "0":
        return None
    try:
        from .. import _native as nat

        return nat
    except ImportError:
        return None


def _from_native(head, path: str) -> GGUFFile:
    version, md, mdt, tlist, alignment, data_offset, file_t = head
    mdt = {k: GGUFValueType(v) for k, v in mdt.items()}
    buf = file_t.numpy()  # zero-copy: the array keeps the mapping alive
    buf.flags.writeable = False  # the pages are mapped read-only
    infos: dict[str, TensorInfo] = {}
    for name, shape, tt, off in tlist:
        infos[name] = TensorInfo(name, tuple(shape), GGMLType(tt), off)
    for t in infos.values():
        if t.ggml_type not in TYPE_TRAITS:
            raise GGUFError(f"tensor {t.name}: unsupported ggml type {t.ggml_type.name}")
        start = data_offset + t.offset
        if start + t.nbytes > buf.shape[0]:
            raise GGUFError(f"tensor {t.name} extends past end of file")
        t.data = buf[start: start + t.nbytes]
    return GGUFFile(path, version, md, mdt, infos, int(alignment), int(data_offset), _mm=file_t)


def read_gguf(path: str | os.PathLike, native: bool | None = None) -> GGUFFile:
    """Memory-map ``path`` and parse its header; tensor data stays in the page cache.  The header is
    parsed by the C++ parser (``_native.gguf_parse``) when it is built, else in Python;
    ``native=False`` or ``BARQ_GGUF_NATIVE=0`` forces the Python parser."""
    path = os.fspath(path)
    nat = _native() if native is not False else None
    if native and nat is None:
        raise ImportError("barq_inference_b200._native is not built (python setup.py build_ext --inplace)")
    if nat is not None:
        try:
            head = nat.gguf_parse(path)
        except ValueError as e:
            msg = str(e)
            raise GGUFError(msg if msg.startswith(path) else f"{path}: {msg}") from None
        try:
            return _from_native(head, path)
        except ValueError as e:
            if isinstance(e, GGUFError):
                raise
            raise GGUFError(f"{path}: {e}") from None
    with open(path, "rb") as f:
        size = os.fstat(f.fileno()).st_size
        if size < 24:
            raise GGUFError(f"{path}: too small for a GGUF header")
        mm = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
    g = _parse(mm, path)
    g._mm = mm
    return g


_SPLIT_RE = re.compile(r"^(?P<base>.*)-(?P<no>\d{5})-of-(?P<count>\d{5})\.gguf$")


def split_paths(path: str | os.PathLike) -> list[str]:
    """All parts of a split GGUF (``name-00001-of-0000N.gguf``), or ``[path]`` for a single file."""
    path = os.fspath(path)
    m = _SPLIT_RE.match(path)
    if not m:
        return [path]
    n = int(m.group("count"))
    return [f"{m.group('base')}-{i:05d}-of-{n:05d}.gguf" for i in range(1, n + 1)]


def read_gguf_split(path: str | os.PathLike) -> GGUFFile:
    """Open a GGUF that may be split into parts (llama.cpp ``gguf-split`` naming and ``split.*``
    keys): metadata comes from the first part, tensors from all of them (each part mmap'd)."""
    parts = split_paths(path)
    first = read_gguf(parts[0])
    count = int(first.metadata.get("split.count", len(parts)))
    if count != len(parts):
        parts = split_paths(parts[0]) if count == len(parts) else parts
        if count != len(parts):
            raise GGUFError(f"{path}: split.count is {count} but {len(parts)} part file(s) were found")
    if count <= 1:
        return first
    maps = [first._mm]
    for i, p in enumerate(parts[1:], start=2):
        g = read_gguf(p)
        no = int(g.metadata.get("split.no", i - 1))
        if no != i - 1:
            raise GGUFError(f"{p}: split.no is {no}, expected {i - 1}")
        dup = set(g.tensors) & set(first.tensors)
        if dup:
            raise GGUFError(f"{p}: tensor(s) {sorted(dup)[:3]} already in an earlier part")
        first.tensors.update(g.tensors)
        maps.append(g._mm)
    first._parts = maps  # keep every part mapped while the tensors are in use
    expected = first.metadata.get("split.tensors.count")
    if expected is not None and int(expected) != len(first.tensors):
        raise GGUFError(f"{path}: {len(first.tensors)} tensors across parts, split.tensors.count says {expected}")
    return first


def read_gguf_bytes(data: bytes) -> GGUFFile:
    return _parse(memoryview(data), "<bytes>")
