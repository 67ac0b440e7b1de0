"""Sampling: host sampler chain, GBNF grammars, JSON mode."""
from .grammar import Grammar, GrammarError, GrammarMatcher, TokenTrie
from .json_mode import JSON_GBNF, schema_to_gbnf, validate_output
from .host_samplers import HostSampler, sample_chain
