"""GGUF / ggml constants: file magic, metadata value types and ggml tensor types.

The numeric ids follow the public GGUF specification (ggml ``ggml_type`` enum and
``gguf_type`` enum), not the reference's private numbering: the reference assigns
non-standard ids to its ik-quants (``barq_core/src/gguf.rs:133-136,157-160``) and
only declares IQ4_NL as an enum tag (``barq_core/src/quant.rs:35``).
"""
from __future__ import annotations

import enum
from dataclasses import dataclass

GGUF_MAGIC = 0x46554747  # b"GGUF" little endian
GGUF_VERSION = 3
GGUF_DEFAULT_ALIGNMENT = 32


class GGUFValueType(enum.IntEnum):
    UINT8 = 0
    INT8 = 1
    UINT16 = 2
    INT16 = 3
    UINT32 = 4
    INT32 = 5
    FLOAT32 = 6
    BOOL = 7
    STRING = 8
    ARRAY = 9
    UINT64 = 10
    INT64 = 11
    FLOAT64 = 12


class GGMLType(enum.IntEnum):
    F32 = 0
    F16 = 1
    Q4_0 = 2
    Q4_1 = 3
    Q5_0 = 6
    Q5_1 = 7
    Q8_0 = 8
    Q8_1 = 9
    Q2_K = 10
    Q3_K = 11
    Q4_K = 12
    Q5_K = 13
    Q6_K = 14
    Q8_K = 15
    IQ2_XXS = 16
    IQ2_XS = 17
    IQ3_XXS = 18
    IQ1_S = 19
    IQ4_NL = 20
    IQ3_S = 21
    IQ2_S = 22
    IQ4_XS = 23
    I8 = 24
    I16 = 25
    I32 = 26
    I64 = 27
    F64 = 28
    IQ1_M = 29
    BF16 = 30
    TQ1_0 = 34
    TQ2_0 = 35
    # ik_llama.cpp extension types (its ``ggml_type`` numbering).  Their rows start with a row
    # scale (``row_meta`` bytes) before the blocks.
    IQ4_KS = 144
    IQ2_KS = 145
    IQ3_KS = 156


@dataclass(frozen=True)
class TypeTraits:
    block_size: int  # elements per block
    type_size: int  # bytes per block
    row_meta: int = 0  # bytes at the start of every row (ik_llama row scale), 0 for ggml types


QK_K = 256

TYPE_TRAITS: dict[GGMLType, TypeTraits] = {
    GGMLType.F32: TypeTraits(1, 4),
    GGMLType.F16: TypeTraits(1, 2),
    GGMLType.BF16: TypeTraits(1, 2),
    GGMLType.F64: TypeTraits(1, 8),
    GGMLType.I8: TypeTraits(1, 1),
    GGMLType.I16: TypeTraits(1, 2),
    GGMLType.I32: TypeTraits(1, 4),
    GGMLType.I64: TypeTraits(1, 8),
    GGMLType.Q4_0: TypeTraits(32, 2 + 16),
    GGMLType.Q4_1: TypeTraits(32, 2 + 2 + 16),
    GGMLType.Q5_0: TypeTraits(32, 2 + 4 + 16),
    GGMLType.Q5_1: TypeTraits(32, 2 + 2 + 4 + 16),
    GGMLType.Q8_0: TypeTraits(32, 2 + 32),
    GGMLType.Q8_1: TypeTraits(32, 4 + 32),
    GGMLType.Q2_K: TypeTraits(QK_K, 16 + 64 + 2 + 2),
    GGMLType.Q3_K: TypeTraits(QK_K, 32 + 64 + 12 + 2),
    GGMLType.Q4_K: TypeTraits(QK_K, 2 + 2 + 12 + 128),
    GGMLType.Q5_K: TypeTraits(QK_K, 2 + 2 + 12 + 32 + 128),
    GGMLType.Q6_K: TypeTraits(QK_K, 128 + 64 + 16 + 2),
    GGMLType.Q8_K: TypeTraits(QK_K, 4 + 256 + 32),
    GGMLType.IQ4_NL: TypeTraits(32, 2 + 16),
    GGMLType.IQ4_XS: TypeTraits(QK_K, 2 + 2 + 4 + 128),
    GGMLType.TQ1_0: TypeTraits(QK_K, 48 + 4 + 2),
    GGMLType.TQ2_0: TypeTraits(QK_K, 64 + 2),
    GGMLType.IQ4_KS: TypeTraits(QK_K, 8 + 128, 4),  # f32 row scale; scales[8], qs[128]
    GGMLType.IQ2_KS: TypeTraits(QK_K, 2 + 4 + 64, 2),  # f16 row scale; extra, scales[4], qs[64]
    GGMLType.IQ3_KS: TypeTraits(QK_K, 2 + 4 + 64 + 32, 2),  # f16 row scale; extra, scales[4], qs[64], qh[32]
}

# ik_llama non-linear codebooks (published format tables): a base half and a shifted half,
# selected per 32-element block.
KVALUES_IQ4K = (-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113,
                -123, -100, -79, -61, -45, -31, -18, -6, 5, 17, 29, 42, 57, 73, 93, 117)
KVALUES_IQ2NL = (-31, -13, 1, 17, -26, -8, 6, 22)
KVALUES_IQ3NL = (-63, -40, -23, -10, 1, 13, 28, 47, -59, -36, -19, -6, 5, 17, 32, 51)

# IQ4_NL / IQ4_XS non-linear 4-bit codebook (published ggml GGUF format table).
KVALUES_IQ4NL = (-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113)

# Reference-level quant names (``barq_core/src/quant.rs:8-48``) mapped onto ggml types
# where a standard GGUF layout exists.
QUANT_NAME_TO_TYPE: dict[str, GGMLType] = {
    "f32": GGMLType.F32,
    "f16": GGMLType.F16,
    "bf16": GGMLType.BF16,
    "q4_0": GGMLType.Q4_0,
    "q4_1": GGMLType.Q4_1,
    "q5_0": GGMLType.Q5_0,
    "q5_1": GGMLType.Q5_1,
    "q8_0": GGMLType.Q8_0,
    "q2_k": GGMLType.Q2_K,
    "q3_k": GGMLType.Q3_K,
    "q4_k": GGMLType.Q4_K,
    "q5_k": GGMLType.Q5_K,
    "q6_k": GGMLType.Q6_K,
    "q8_k": GGMLType.Q8_K,
    "iq4_nl": GGMLType.IQ4_NL,
    "iq4_xs": GGMLType.IQ4_XS,
    "tq1_0": GGMLType.TQ1_0,
    "tq2_0": GGMLType.TQ2_0,
    "iq4_ks": GGMLType.IQ4_KS,
    "iq3_ks": GGMLType.IQ3_KS,
    "iq2_ks": GGMLType.IQ2_KS,
}


def row_nbytes(t: GGMLType, ne0: int) -> int:
    """Bytes of one row of ``ne0`` elements (row scale included for ik_llama types)."""
    tr = TYPE_TRAITS[GGMLType(t)]
    if ne0 % tr.block_size:
        raise ValueError(f"{GGMLType(t).name}: row of {ne0} elements not a multiple of block {tr.block_size}")
    return tr.row_meta + ne0 // tr.block_size * tr.type_size


def type_nbytes(t: GGMLType, n_elements: int, ne0: int | None = None) -> int:
    """Bytes of ``n_elements`` values; row-scaled types also need the row length ``ne0``."""
    tr = TYPE_TRAITS[GGMLType(t)]
    if n_elements % tr.block_size:
        raise ValueError(f"{GGMLType(t).name}: {n_elements} elements not a multiple of block {tr.block_size}")
    if tr.row_meta:
        if ne0 is None:
            raise ValueError(f"{GGMLType(t).name}: row length needed (per-row scale)")
        return n_elements // ne0 * row_nbytes(t, ne0)
    return n_elements // tr.block_size * tr.type_size


def bits_per_weight(t: GGMLType) -> float:
    tr = TYPE_TRAITS[GGMLType(t)]
    return tr.type_size * 8.0 / tr.block_size
