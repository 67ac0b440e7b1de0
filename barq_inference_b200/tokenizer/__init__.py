"""Tokenizers from GGUF metadata and chat templates."""
from .gguf_tokenizer import GGUFTokenizer, StreamDecoder, synthetic_tokenizer
from .chat_template import ChatTemplate, parse_role
