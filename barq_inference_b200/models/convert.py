"""GGUF -> GGUF requantization (``barq convert``).

Parity: ``convert`` (``cli/src/main.rs:834-884``) and ``quantize_model_ik`` / ``repack_model_cpu``
(``quant/src/ik_quant.rs:275-297``), which write a private ``IKQ1`` archive.  This writes a standard
GGUF: every 2-D+ weight is dequantized (ggml-spec oracle) and requantized to the requested type
(rows that do not divide the block size fall back like llama.cpp's quantizer); norms, biases and
1-D tensors keep their type; metadata is copied.
"""
from __future__ import annotations

import numpy as np
import torch

from ..gguf import GGMLType, GGUFWriter, dequantize, quantize
from ..gguf import read_gguf_split as read_gguf
from .weights import fallback_type

KEEP_SUFFIXES = ("_norm.weight", ".bias", "norm.weight")


def convert_gguf(src: str, dst: str, target: GGMLType, keep_output_type: str | None = None,
                 device: str | None = None) -> None:
    g = read_gguf(src)
    w = GGUFWriter(dst)
    for k, v in g.metadata.items():
        if k == "general.alignment":
            continue
        w.add(k, v, g.metadata_types.get(k))
    dev = device or ("cuda" if torch.cuda.is_available() else "cpu")
    for name, ti in g.tensors.items():
        shape = ti.torch_shape
        if len(shape) < 2 or name.endswith(KEEP_SUFFIXES) or "ffn_gate_inp" in name:
            w.add_tensor(name, np.array(ti.data), ti.ggml_type, shape)
            continue
        t = target
        if name == "output.weight" and keep_output_type:
            t = GGMLType[keep_output_type.upper()] if keep_output_type.lower() != "keep" else ti.ggml_type
        t = fallback_type(t, shape[-1])
        if t == ti.ggml_type:
            w.add_tensor(name, np.array(ti.data), t, shape)
            continue
        x = torch.from_numpy(dequantize(np.array(ti.data), ti.ggml_type, shape)).to(dev)
        q = quantize(x.reshape(-1, shape[-1]), t).cpu().numpy()
        w.add_tensor(name, q, t, shape)
    w.write()
