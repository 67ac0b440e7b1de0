"""GGUF v3 writer.

Used by ``convert`` (GGUF -> GGUF requantization) and by the random-init model generator
that produces benchmark checkpoints.  The reference writes a private ``IKQ1`` archive
instead (``quant/src/ik_quant.rs:136,187``); here the output is a standard GGUF file.
"""
from __future__ import annotations

import os
import struct
from typing import Any, Iterable

import numpy as np

from .constants import GGUF_DEFAULT_ALIGNMENT, GGUF_MAGIC, GGUF_VERSION, TYPE_TRAITS, GGMLType, GGUFValueType, row_nbytes


def _infer_vt(v: Any) -> GGUFValueType:
    if isinstance(v, bool):
        return GGUFValueType.BOOL
    if isinstance(v, int):
        return GGUFValueType.UINT32 if 0 <= v < 2**32 else GGUFValueType.INT64
    if isinstance(v, float):
        return GGUFValueType.FLOAT32
    if isinstance(v, str):
        return GGUFValueType.STRING
    if isinstance(v, (list, tuple, np.ndarray)):
        return GGUFValueType.ARRAY
    raise TypeError(f"cannot infer GGUF type for {type(v)}")


_FMT = {
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

_NP = {
    GGUFValueType.UINT8: "<u1",
    GGUFValueType.INT8: "<i1",
    GGUFValueType.UINT16: "<u2",
    GGUFValueType.INT16: "<i2",
    GGUFValueType.UINT32: "<u4",
    GGUFValueType.INT32: "<i4",
    GGUFValueType.FLOAT32: "<f4",
    GGUFValueType.BOOL: "?",
    GGUFValueType.UINT64: "<u8",
    GGUFValueType.INT64: "<i8",
    GGUFValueType.FLOAT64: "<f8",
}


def _enc_str(s: str) -> bytes:
    b = s.encode("utf-8")
    return struct.pack("<Q", len(b)) + b


def _enc_value(v: Any, vt: GGUFValueType, elem_vt: GGUFValueType | None = None) -> bytes:
    if vt == GGUFValueType.STRING:
        return _enc_str(v)
    if vt == GGUFValueType.ARRAY:
        seq = list(v) if not isinstance(v, np.ndarray) else v
        if elem_vt is None:
            if len(seq) == 0:
                elem_vt = GGUFValueType.UINT32
            elif isinstance(seq, np.ndarray):
                elem_vt = {
                    np.dtype(np.float32): GGUFValueType.FLOAT32,
                    np.dtype(np.int32): GGUFValueType.INT32,
                    np.dtype(np.uint32): GGUFValueType.UINT32,
                    np.dtype(np.int64): GGUFValueType.INT64,
                    np.dtype(np.uint8): GGUFValueType.UINT8,
                    np.dtype(np.int8): GGUFValueType.INT8,
                    np.dtype(np.float64): GGUFValueType.FLOAT64,
                    np.dtype(np.bool_): GGUFValueType.BOOL,
                }[seq.dtype]
            else:
                elem_vt = _infer_vt(seq[0])
                if elem_vt == GGUFValueType.UINT32 and any((not isinstance(x, bool)) and isinstance(x, int) and x < 0 for x in seq):
                    elem_vt = GGUFValueType.INT32
        out = struct.pack("<IQ", int(elem_vt), len(seq))
        if elem_vt in _NP:
            out += np.asarray(seq).astype(_NP[elem_vt]).tobytes()
        else:
            out += b"".join(_enc_value(x, elem_vt) for x in seq)
        return out
    return struct.pack(_FMT[vt], v)


class GGUFWriter:
    """Collects metadata and packed tensors, then writes one GGUF v3 file."""

    def __init__(self, path: str | os.PathLike, arch: str | None = None, alignment: int = GGUF_DEFAULT_ALIGNMENT):
        self.path = os.fspath(path)
        self.alignment = alignment
        self.kv: list[tuple[str, Any, GGUFValueType, GGUFValueType | None]] = []
        self.tensors: list[tuple[str, tuple[int, ...], GGMLType, np.ndarray]] = []
        if arch is not None:
            self.add("general.architecture", arch)
        if alignment != GGUF_DEFAULT_ALIGNMENT:
            self.add("general.alignment", alignment, GGUFValueType.UINT32)

    def add(self, key: str, value: Any, vt: GGUFValueType | None = None, elem_vt: GGUFValueType | None = None) -> None:
        self.kv.append((key, value, vt if vt is not None else _infer_vt(value), elem_vt))

    def add_tensor(self, name: str, data: np.ndarray, ggml_type: GGMLType, shape: Iterable[int]) -> None:
        """``shape`` is row-major (outermost first); ``data`` holds the packed bytes."""
        shape = tuple(int(s) for s in shape)
        ne = tuple(reversed(shape))
        n = int(np.prod(shape)) if shape else 1
        tr = TYPE_TRAITS[ggml_type]
        if ne[0] % tr.block_size:
            raise ValueError(f"{name}: row length {ne[0]} not a multiple of {tr.block_size}")
        raw = np.ascontiguousarray(data).view(np.uint8).reshape(-1)
        want = n // ne[0] * row_nbytes(ggml_type, ne[0]) if ne else tr.type_size
        if raw.size != want:
            raise ValueError(f"{name}: {raw.size} bytes given, {want} expected for {ggml_type.name}{shape}")
        self.tensors.append((name, ne, GGMLType(ggml_type), raw))

    def write(self) -> None:
        a = self.alignment
        header = struct.pack("<IIQQ", GGUF_MAGIC, GGUF_VERSION, len(self.tensors), len(self.kv))
        body = bytearray()
        for key, v, vt, evt in self.kv:
            body += _enc_str(key) + struct.pack("<I", int(vt)) + _enc_value(v, vt, evt)
        off = 0
        offsets = []
        for name, ne, tt, raw in self.tensors:
            offsets.append(off)
            off += (raw.size + a - 1) // a * a
        for (name, ne, tt, raw), o in zip(self.tensors, offsets):
            body += _enc_str(name) + struct.pack("<I", len(ne)) + b"".join(struct.pack("<Q", d) for d in ne)
            body += struct.pack("<IQ", int(tt), o)
        with open(self.path, "wb") as f:
            f.write(header)
            f.write(body)
            pos = len(header) + len(body)
            pad = (pos + a - 1) // a * a - pos
            f.write(b"\0" * pad)
            for (name, ne, tt, raw), o in zip(self.tensors, offsets):
                f.write(memoryview(raw))
                p = (raw.size + a - 1) // a * a - raw.size
                if p:
                    f.write(b"\0" * p)
