"""Log-probabilities of sampled tokens for the API's ``logprobs`` / ``top_logprobs``.

The value is the log-softmax of the raw logits at the sampled token (before temperature, top-k/p,
penalties or grammar masks: the model's own distribution, as OpenAI-style APIs report it), plus the
``top_logprobs`` most likely tokens.  Only the rows of sequences that asked for it are computed.
"""
from __future__ import annotations

import torch


def record_logprobs(logits: torch.Tensor, rows: list[int], ids: list[int], seqs: list) -> None:
    """Append to ``seqs[r].logprobs`` / ``.top_logprobs`` for every r in ``rows``; ``logits`` holds one
    row per sequence ([len(seqs), V]) and ``ids`` the sampled tokens."""
    if not rows:
        return
    dev = logits.device
    lsm = torch.log_softmax(logits[torch.tensor(rows, device=dev)].float(), dim=-1)
    chosen = lsm.gather(1, torch.tensor([[ids[r]] for r in rows], device=dev)).squeeze(1).cpu().tolist()
    k = max(seqs[r].params.top_logprobs for r in rows)
    top_v = top_i = None
    if k > 0:
        tv, ti = lsm.topk(min(k, lsm.shape[1]), dim=-1)
        top_v, top_i = tv.cpu().tolist(), ti.cpu().tolist()
    for j, r in enumerate(rows):
        s = seqs[r]
        s.logprobs.append(chosen[j])
        n = s.params.top_logprobs
        s.top_logprobs.append(list(zip(top_i[j][:n], top_v[j][:n])) if n and top_i is not None else [])
