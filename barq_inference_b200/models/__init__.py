"""Model families: config extraction, GGUF tensor plans, reference forward and device runners."""
from .config import ModelConfig, PRESETS, preset, config_from_gguf
from .weights import QuantPolicy, POLICIES, PackedTensor, tensor_plan, random_tensors, write_gguf, tensors_from_gguf, config_metadata
