"""GGUF checkpoint format: reader, writer, ggml block quantizers and dequantizers."""
from .constants import GGMLType, GGUFValueType, TYPE_TRAITS, QK_K, KVALUES_IQ4NL, type_nbytes, row_nbytes, bits_per_weight, QUANT_NAME_TO_TYPE
from .reader import GGUFFile, TensorInfo, GGUFError, read_gguf, read_gguf_bytes, read_gguf_split, split_paths
from .writer import GGUFWriter
from .dequant import dequantize, supported_dequant_types
from .quantize import quantize, QUANTIZERS
