"""Serving benchmark: drive an OpenAI-compatible server (``barq-http``, ``barq http-server`` or any
other) with concurrent streaming requests and report latency and throughput as the client sees them.

Per request: time to first token (TTFT), inter-token latency (ITL: gaps between streamed chunks after
the first), end-to-end latency and output tokens (from ``stream_options.include_usage``, else the
chunk count).  Summary: request and output-token throughput over the wall time, and p50 / p90 /
p99 of TTFT, ITL and latency.  Requests are released either all at once (bounded by
``concurrency``) or as a Poisson process of ``rate`` requests per second.

The reference measures its engine in-process (``cli/src/benchmark.rs``); this client-side view of
a running server is what a deployment is judged by.
"""
from __future__ import annotations

import asyncio
import json
import random
import time
from dataclasses import dataclass, field


@dataclass
class RequestStats:
    ok: bool = False
    error: str = ""
    ttft_s: float = 0.0
    latency_s: float = 0.0
    itl_s: list[float] = field(default_factory=list)
    output_tokens: int = 0


def _pct(xs: list[float], p: float) -> float:
    if not xs:
        return 0.0
    s = sorted(xs)
    return s[min(len(s) - 1, max(0, int(round(p / 100.0 * len(s) + 0.5)) - 1))]


def _prompt(i: int, words: int, seed: int) -> str:
    rng = random.Random(seed * 1000003 + i)
    vocab = ["alpha", "beta", "gamma", "delta", "epsilon", "zeta", "eta", "theta", "iota", "kappa", "lambda",
             "mu", "nu", "xi", "omicron", "pi", "rho", "sigma", "tau", "upsilon"]
    return " ".join(rng.choice(vocab) for _ in range(words))


async def _one(session, url: str, body: dict) -> RequestStats:
    st = RequestStats()
    t0 = time.perf_counter()
    last = None
    try:
        async with session.post(url, json=body) as resp:
            if resp.status != 200:
                st.error = f"HTTP {resp.status}: {(await resp.text())[:200]}"
                return st
            buf = b""
            async for chunk in resp.content.iter_any():
                buf += chunk
                while b"\n\n" in buf:
                    event, buf = buf.split(b"\n\n", 1)
                    if not event.startswith(b"data: "):
                        continue
                    data = event[6:]
                    if data == b"[DONE]":
                        continue
                    obj = json.loads(data)
                    if obj.get("usage"):
                        st.output_tokens = int(obj["usage"].get("completion_tokens", st.output_tokens))
                    ch = (obj.get("choices") or [{}])[0]
                    text = ch.get("text") or (ch.get("delta") or {}).get("content") or obj.get("output") or ""
                    if not text:
                        continue
                    now = time.perf_counter()
                    if last is None:
                        st.ttft_s = now - t0
                    else:
                        st.itl_s.append(now - last)
                    last = now
            st.latency_s = time.perf_counter() - t0
            if st.output_tokens == 0:  # no usage chunk from the server: count the streamed chunks
                st.output_tokens = len(st.itl_s) + (1 if last is not None else 0)
            st.ok = last is not None
            if not st.ok:
                st.error = "no tokens streamed"
    except Exception as e:  # noqa: BLE001 - a failed request is counted, the run goes on
        st.error = f"{type(e).__name__}: {e}"
    return st


async def run(url: str, n_requests: int = 64, concurrency: int = 16, prompt_words: int = 64,
              max_tokens: int = 128, rate: float = 0.0, chat: bool = False, model: str = "barq",
              seed: int = 0, temperature: float = 0.0, api_key: str | None = None) -> dict:
    """Benchmark ``url`` (the server's base URL, e.g. ``http://127.0.0.1:8080``); returns the summary."""
    import aiohttp

    path = "/v1/chat/completions" if chat else "/v1/completions"
    sem = asyncio.Semaphore(max(1, concurrency))
    rng = random.Random(seed)
    timeout = aiohttp.ClientTimeout(total=None, sock_read=600)

    headers = {"Authorization": f"Bearer {api_key}"} if api_key else None
    async with aiohttp.ClientSession(timeout=timeout, headers=headers) as session:
        async def task(i: int, delay: float) -> RequestStats:
            if delay:
                await asyncio.sleep(delay)
            text = _prompt(i, prompt_words, seed)
            body = {"model": model, "max_tokens": max_tokens, "temperature": temperature, "stream": True,
                    "stream_options": {"include_usage": True}}
            if chat:
                body["messages"] = [{"role": "user", "content": text}]
            else:
                body["prompt"] = text
            async with sem:
                return await _one(session, url.rstrip("/") + path, body)

        t0 = time.perf_counter()
        delays, t = [], 0.0
        for _ in range(n_requests):
            delays.append(t)
            if rate > 0:
                t += rng.expovariate(rate)
        stats = await asyncio.gather(*(task(i, d) for i, d in enumerate(delays)))
        wall = time.perf_counter() - t0
    ok = [s for s in stats if s.ok]
    itl = [x for s in ok for x in s.itl_s]
    out_tok = sum(s.output_tokens for s in ok)
    ms = lambda xs, p: round(_pct(xs, p) * 1e3, 3)  # noqa: E731
    return {
        "url": url, "route": path, "requests": n_requests, "completed": len(ok), "failed": len(stats) - len(ok),
        "errors": sorted({s.error for s in stats if s.error})[:5],
        "concurrency": concurrency, "rate_rps": rate, "wall_s": round(wall, 3),
        "request_throughput_rps": round(len(ok) / wall, 3) if wall else 0.0,
        "output_token_throughput_tok_s": round(out_tok / wall, 2) if wall else 0.0,
        "output_tokens": out_tok,
        **{f"ttft_p{p}_ms": ms([s.ttft_s for s in ok], p) for p in (50, 90, 99)},
        **{f"itl_p{p}_ms": ms(itl, p) for p in (50, 90, 99)},
        **{f"latency_p{p}_ms": ms([s.latency_s for s in ok], p) for p in (50, 90, 99)},
    }
