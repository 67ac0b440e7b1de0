"""Sampling parameters of a request body, shared by the OpenAI HTTP server and the UDS server."""
from __future__ import annotations

from ..engine.sampling_params import SamplingParams

DEFAULTS = dict(max_tokens=128, temperature=0.8, top_k=40, top_p=0.95)


def sampling_params_from_request(body: dict, max_key: str = "max_tokens") -> SamplingParams:
    """SamplingParams of an OpenAI-style request body (HTTP routes and UDS frames share it).

    Defaults follow the reference's server handler (``cli/src/server.rs``): max_tokens 128,
    temperature 0.8, top_k 40, top_p 0.95.  ``response_format`` selects JSON mode or a JSON
    schema, ``grammar`` a GBNF grammar; ValueError on invalid values."""
    mt = body.get(max_key)
    if mt is None:
        mt = body.get("max_output_tokens", body.get("max_tokens", DEFAULTS["max_tokens"]))
    p = SamplingParams(
        max_tokens=int(mt),
        temperature=float(body.get("temperature", DEFAULTS["temperature"])),
        top_k=int(body.get("top_k", DEFAULTS["top_k"])),
        top_p=float(body.get("top_p", DEFAULTS["top_p"])),
        min_p=float(body.get("min_p", 0.0)),
        repetition_penalty=float(body.get("repetition_penalty", 1.0)),
        frequency_penalty=float(body.get("frequency_penalty", 0.0)),
        presence_penalty=float(body.get("presence_penalty", 0.0)),
        seed=int(body.get("seed", 0) or 0),
    )
    # chat: logprobs (bool) + top_logprobs (int); completions: logprobs = number of alternatives
    lp = body.get("logprobs")
    if isinstance(lp, bool) or lp is None:
        p.logprobs = bool(lp)
        p.top_logprobs = int(body.get("top_logprobs", 0) or 0) if p.logprobs else 0
    elif isinstance(lp, int):
        p.logprobs, p.top_logprobs = True, lp
    else:
        raise ValueError("logprobs must be a boolean or an integer")
    if not 0 <= p.top_logprobs <= 20:
        raise ValueError("top_logprobs must be between 0 and 20")
    if p.max_tokens < 1:
        raise ValueError("max_tokens must be >= 1")
    rf = body.get("response_format") or {}
    if isinstance(rf, dict):
        if rf.get("type") == "json_object":
            p.json_mode = True
        elif rf.get("type") == "json_schema":
            js = rf.get("json_schema") or {}
            p.json_schema = js.get("schema", js) if isinstance(js, dict) else None
            p.json_mode = True
    if body.get("grammar"):
        p.grammar = str(body["grammar"])
    return p
