"""``IKQ1`` archive: the container ``barq convert`` writes for the ik quant types.

Parity: ``write_ikq_archive`` / ``quantize_model_ik`` / ``repack_model_cpu``
(``quant/src/ik_quant.rs:135-305``).  The byte layout is kept identical to the reference's so
archives move between the two (all integers little endian):

    "IKQ1" | u32 version=1 | u32 archive quant id | u32 n_tensors | u32 n_meta
    n_meta x (str key, str value)                      str = u32 length + UTF-8 bytes
    n_tensors x (str name | u32 n_dims | n_dims x u64 dim | u32 source ggml type
                 | u32 quant id | u64 n_bytes | bytes)

Quant ids: 1 IQ4_KS, 2 IQ3_KS, 3 IQ2_KS, 4 Q4_K_R4 (the reference's numbering); this module adds
0 = raw f32 for tensors that stay unquantized (norms, biases, 1-D tensors), which the reference
quantizes as well.  Metadata values are written as JSON ``{"t": gguf value type, "v": value}`` so
that :func:`ikq_to_gguf` restores typed GGUF metadata; the reference writes Rust ``Debug`` text.
IQ*_KS payloads are the row-scaled ik_llama rows of :mod:`.ik_quants`; Q4_K_R4 payloads are
:func:`~.ik_quants.repack_q4_k_r4` groups.
"""
from __future__ import annotations

import json
import struct
from dataclasses import dataclass

import numpy as np
import torch

from .constants import GGMLType, GGUFValueType
from .ik_quants import repack_q4_k_r4, unpack_q4_k_r4

IKQ_MAGIC = b"IKQ1"
IKQ_VERSION = 1
IKQ_RAW, IKQ_IQ4_KS, IKQ_IQ3_KS, IKQ_IQ2_KS, IKQ_Q4_K_R4 = 0, 1, 2, 3, 4
IKQ_NAMES = {"iq4_ks": IKQ_IQ4_KS, "iq3_ks": IKQ_IQ3_KS, "iq2_ks": IKQ_IQ2_KS, "q4_k_r4": IKQ_Q4_K_R4}
_IKQ_TO_GGML = {IKQ_IQ4_KS: GGMLType.IQ4_KS, IKQ_IQ3_KS: GGMLType.IQ3_KS, IKQ_IQ2_KS: GGMLType.IQ2_KS}
KEEP_SUFFIXES = ("_norm.weight", ".bias", "norm.weight")


@dataclass
class IKQTensor:
    name: str
    shape: tuple[int, ...]  # row-major (outermost first)
    src_type: int
    quant: int
    data: np.ndarray  # uint8


@dataclass
class IKQArchive:
    quant: int
    metadata: dict
    metadata_types: dict
    tensors: dict[str, IKQTensor]


def _s(b: bytes) -> bytes:
    return struct.pack("<I", len(b)) + b


def write_ikq(path: str, quant: int, metadata: dict, metadata_types: dict, tensors: list[IKQTensor],
              extra: dict | None = None) -> None:
    meta = [(k, json.dumps({"t": int(metadata_types.get(k, GGUFValueType.STRING)), "v": _jsonable(v)}))
            for k, v in metadata.items()]
    for k, v in (extra or {}).items():
        meta.append((k, json.dumps({"t": int(GGUFValueType.STRING), "v": str(v)})))
    with open(path, "wb") as f:
        f.write(IKQ_MAGIC + struct.pack("<IIII", IKQ_VERSION, quant, len(tensors), len(meta)))
        for k, v in meta:
            f.write(_s(k.encode()) + _s(v.encode()))
        for t in tensors:
            dims = tuple(reversed(t.shape))  # ggml order, innermost first
            f.write(_s(t.name.encode()) + struct.pack("<I", len(dims)) + struct.pack(f"<{len(dims)}Q", *dims))
            raw = np.ascontiguousarray(t.data).view(np.uint8).reshape(-1)
            f.write(struct.pack("<IIQ", int(t.src_type), t.quant, raw.size))
            f.write(raw.tobytes())


def _jsonable(v):
    if isinstance(v, np.ndarray):
        return v.tolist()
    if isinstance(v, (bytes, bytearray)):
        return v.decode("utf-8", "replace")
    if isinstance(v, (list, tuple)):
        return [_jsonable(x) for x in v]
    if isinstance(v, np.generic):
        return v.item()
    return v


def read_ikq(path: str) -> IKQArchive:
    buf = memoryview(open(path, "rb").read())
    pos = 0

    def take(n):
        nonlocal pos
        if pos + n > len(buf):
            raise ValueError(f"{path}: truncated IKQ archive")
        out = buf[pos:pos + n]
        pos += n
        return out

    def u32():
        return struct.unpack("<I", take(4))[0]

    def string():
        return bytes(take(u32())).decode()

    if bytes(take(4)) != IKQ_MAGIC:
        raise ValueError(f"{path}: not an IKQ1 archive")
    version, quant, n_t, n_m = (u32() for _ in range(4))
    if version != IKQ_VERSION:
        raise ValueError(f"{path}: IKQ version {version}")
    md, mdt = {}, {}
    for _ in range(n_m):
        k, v = string(), string()
        try:
            j = json.loads(v)
            md[k], mdt[k] = j["v"], GGUFValueType(j["t"])
        except (ValueError, KeyError, TypeError):  # an archive written with plain text values
            md[k], mdt[k] = v, GGUFValueType.STRING
    ts = {}
    for _ in range(n_t):
        name = string()
        nd = u32()
        dims = struct.unpack(f"<{nd}Q", take(8 * nd))
        src, q = u32(), u32()
        n = struct.unpack("<Q", take(8))[0]
        ts[name] = IKQTensor(name, tuple(reversed(dims)), src, q, np.frombuffer(take(n), np.uint8))
    return IKQArchive(quant, md, mdt, ts)


def gguf_to_ikq(src: str, dst: str, quant_name: str, device: str | None = None) -> None:
    """Requantize every weight matrix of a GGUF (split files too) into an IKQ1 archive."""
    from . import dequantize, quantize, read_gguf_split

    quant = IKQ_NAMES[quant_name.lower()]
    g = read_gguf_split(src)
    dev = device or ("cuda" if torch.cuda.is_available() else "cpu")
    out = []
    for name, ti in g.tensors.items():
        shape = ti.torch_shape
        x = torch.from_numpy(dequantize(np.array(ti.data), ti.ggml_type, shape)).reshape(-1, shape[-1])
        rows = x.shape[0]
        ok = len(shape) >= 2 and not name.endswith(KEEP_SUFFIXES) and "ffn_gate_inp" not in name \
            and shape[-1] % 256 == 0 and (quant != IKQ_Q4_K_R4 or rows % 4 == 0)
        if not ok:
            out.append(IKQTensor(name, shape, ti.ggml_type, IKQ_RAW, x.numpy().astype("<f4").view(np.uint8)))
            continue
        if quant == IKQ_Q4_K_R4:
            q = quantize(x.to(dev), GGMLType.Q4_K).cpu().numpy()
            data = repack_q4_k_r4(q)
        else:
            data = quantize(x.to(dev), _IKQ_TO_GGML[quant]).cpu().numpy()
        out.append(IKQTensor(name, shape, ti.ggml_type, quant, data))
    extra = {"ik.quant_type": quant_name.lower()}
    md = {k: v for k, v in g.metadata.items() if k != "general.alignment"}
    write_ikq(dst, quant, md, g.metadata_types, out, extra)


def ikq_to_gguf(src: str, dst: str) -> None:
    """Write an IKQ1 archive back as a GGUF: IQ*_KS stay ik types (the loader requantizes them for
    the device), Q4_K_R4 unpacks to Q4_K exactly, raw tensors become F32."""
    from .writer import GGUFWriter

    a = read_ikq(src)
    w = GGUFWriter(dst)
    for k, v in a.metadata.items():
        if k.startswith("ik."):
            continue
        w.add(k, v, a.metadata_types.get(k))
    for t in a.tensors.values():
        rows = int(np.prod(t.shape[:-1])) if len(t.shape) > 1 else 1
        if t.quant == IKQ_RAW:
            w.add_tensor(t.name, t.data, GGMLType.F32, t.shape)
        elif t.quant == IKQ_Q4_K_R4:
            w.add_tensor(t.name, unpack_q4_k_r4(t.data, rows), GGMLType.Q4_K, t.shape)
        else:
            w.add_tensor(t.name, t.data, _IKQ_TO_GGML[t.quant], t.shape)
    w.write()
