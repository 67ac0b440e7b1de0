"""``barq`` command line: run, chat, benchmark, info, convert, server, http-server, make-random-gguf,
metal-info, wasm-info.

Parity: the reference's clap CLI (``cli/src/main.rs:39-246``) — global ``--verbose/-v``,
``--threads/-t``, ``--cuda-graphs``, ``--flash-attn``, ``--preset``; ``run`` with ``--model/-m``,
``--prompt``, ``--max-tokens 128``, ``--temperature 0.8``, ``--top-k 40``, ``--top-p 0.95``,
``--context-size 2048``, ``--speculative``, ``--draft-model``, ``--draft-max 16``,
``--speculation-preset``, ``--json``, ``--mla``, ``--fmoe``, ``--ser``; ``benchmark`` with
``--iterations 10 --prompt-length 512 --gen-length 128``; ``convert --input --output --quantize``;
``server`` (UDS) and ``http-server --host 0.0.0.0 --port 8000 --rate-limit-rpm 60``.  The reference's
``chat`` is a TODO and its ``--speculative``/``--fmoe``/``--ser`` flags only log; here they work.
New flags: ``--device``, ``--kv-dtype``, ``--max-batch``, ``--tp``, ``--prefix-cache``.
"""
from __future__ import annotations

import argparse
import json
import logging
import os
import statistics
import sys
import time

log = logging.getLogger("barq")


# ------------------------------------------------------------------ model loading
def load(args, need_engine: bool = True):
    """Returns (engine, tokenizer, chat_template, metadata)."""
    from .gguf import read_gguf_split as read_gguf
    from .models.config import attach_rope_factors, config_from_gguf
    from .models.weights import tensors_from_gguf
    from .tokenizer import ChatTemplate, GGUFTokenizer, synthetic_tokenizer

    g = read_gguf(args.model)
    md = g.metadata
    cfg = attach_rope_factors(config_from_gguf(md, set(g.tensors)), g)
    if getattr(args, "context_size", None):
        cfg.max_ctx = min(cfg.max_ctx, int(args.context_size)) if cfg.max_ctx else int(args.context_size)
    try:
        tok = GGUFTokenizer.from_metadata(md)
    except ValueError:
        tok = synthetic_tokenizer(cfg.vocab)
    tmpl = ChatTemplate.for_arch(cfg.arch, md)
    if not need_engine:
        return None, tok, tmpl, md
    tensors = tensors_from_gguf(g, device="cpu")
    device = getattr(args, "device", None) or ("cuda" if _cuda() else "cpu")
    ser = 0.2 if getattr(args, "ser", False) else 0.0
    if device == "cpu":
        from .engine.cpu_engine import CPUEngine

        eng = CPUEngine(cfg, tensors, max_model_len=cfg.max_ctx, ser_threshold=ser)
    else:
        from .engine.engine import Engine, EngineConfig

        preset = getattr(args, "preset", None)
        tp = int(getattr(args, "tp", 1) or 1)
        if tp > 1:  # one process per GPU under torchrun: this rank's GPU
            import os

            import torch

            local = int(os.environ.get("LOCAL_RANK", "0"))
            torch.cuda.set_device(local)
            device = f"cuda:{local}"
        pp = int(getattr(args, "pp", 1) or 1)
        if pp > 1:  # (with --tp too: a tp x pp grid, global rank = stage * tp + tensor rank)
            import os

            import torch

            local = int(os.environ.get("LOCAL_RANK", "0"))
            torch.cuda.set_device(local)
            device = f"cuda:{local}"
        kw = dict(max_model_len=cfg.max_ctx, device=device, ser_threshold=ser,
                  fused_moe=not getattr(args, "no_fmoe", False), tp=tp, pp=pp,
                  fused_comm=getattr(args, "comm", "fused") != "nccl",
                  block_size=int(getattr(args, "block_size", 16) or 16),
                  kv_dtype=getattr(args, "kv_dtype", "fp16") or "fp16",
                  max_num_seqs=getattr(args, "max_batch", 64) or 64,
                  prefix_caching=bool(getattr(args, "prefix_cache", False) or getattr(args, "prompt_cache", None)),
                  kv_cache_gb=float(getattr(args, "kv_cache_gb", 8.0) or 8.0),
                  max_waiting=int(getattr(args, "max_waiting", 0) or 0))
        if getattr(args, "cuda_graphs", None) is not None:
            kw["cuda_graphs"] = bool(args.cuda_graphs)
        ec = EngineConfig.preset(preset, **kw) if preset else EngineConfig(**kw)
        eng = Engine(cfg, tensors, ec)
        if getattr(args, "mla", False) and not cfg.is_mla:
            log.warning("--mla: %s has no MLA attention; flag ignored", cfg.arch)
    eng.tokenizer = tok
    return eng, tok, tmpl, md


def _cuda() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


def _params(args):
    from .engine.sampling_params import SamplingParams

    return SamplingParams(max_tokens=args.max_tokens, temperature=args.temperature, top_k=args.top_k,
                          top_p=args.top_p, min_p=getattr(args, "min_p", 0.0),
                          repetition_penalty=getattr(args, "repeat_penalty", 1.0),
                          seed=getattr(args, "seed", 0), json_mode=bool(getattr(args, "json", False)))


# ------------------------------------------------------------------ subcommands
def cmd_run(args) -> int:
    from .tokenizer import StreamDecoder

    eng, tok, tmpl, _ = load(args)
    if args.prompt_ids:
        ids = [int(x) for x in args.prompt_ids.split(",") if x.strip()]
    else:
        text = args.prompt
        if args.chat_format:
            text = tmpl.render([{"role": "user", "content": args.prompt}])
        ids = tok.encode(text)
    params = _params(args)
    if args.speculative or args.draft_model or args.lookup_decoding:
        from .engine.speculative import SpeculativeDecoder, SpeculativeConfig

        draft = None  # --lookup-decoding: drafts from n-grams of the context, no draft model
        if not args.lookup_decoding:
            draft_args = argparse.Namespace(**{**vars(args), "model": args.draft_model or args.model})
            draft, _, _, _ = load(draft_args)
        sc = SpeculativeConfig.preset(args.speculation_preset, draft_max=args.draft_max)
        out = SpeculativeDecoder(eng, draft, sc, lookup_ngram=args.lookup_ngram).generate(ids, params)
        sys.stdout.write(tok.decode(out.tokens) + "\n")
        log.info("speculative: acceptance %.2f", out.acceptance_rate)
        return 0
    pc = getattr(args, "prompt_cache", None)
    if pc and os.path.exists(pc):
        from .engine.session import import_session

        try:
            log.info("prompt cache %s: %d tokens reusable", pc, import_session(eng, pc))
        except (ValueError, NotImplementedError) as e:
            log.warning("prompt cache %s not used: %s", pc, e)
    dec = StreamDecoder(tok)
    t0 = time.perf_counter()
    first = [None]

    def on_token(seq, t):
        if t < 0 or (t in eng.cfg.eos_ids):
            return
        if first[0] is None:
            first[0] = time.perf_counter()
        sys.stdout.write(dec.push(t))
        sys.stdout.flush()

    seq = eng.add_request(ids, params, on_token=on_token)
    while eng.has_work():
        eng.step()
    sys.stdout.write(dec.flush() + "\n")
    dt = time.perf_counter() - t0
    if args.json:
        from .sampling.json_mode import validate_output

        if not validate_output(tok.decode(seq.output)):
            log.warning("output is not valid JSON")
    n = len(seq.output)
    log.info("%d prompt tokens, %d generated in %.2fs (%.1f tok/s, TTFT %.1f ms)", len(ids), n, dt, n / max(dt, 1e-9),
             ((first[0] or t0) - t0) * 1e3)
    if pc:
        from .engine.session import export_session

        try:
            export_session(eng, ids, pc)
            log.info("prompt cache written to %s", pc)
        except (ValueError, NotImplementedError) as e:
            log.warning("prompt cache not written: %s", e)
    return 0


def cmd_chat(args) -> int:
    from .tokenizer import StreamDecoder

    eng, tok, tmpl, _ = load(args)
    history = []
    if args.system_prompt:
        history.append({"role": "system", "content": args.system_prompt})
    params = _params(args)
    print("barq chat — empty line or /exit to quit")
    while True:
        try:
            line = input("> ")
        except EOFError:
            break
        if not line.strip() or line.strip() in ("/exit", "/quit"):
            break
        history.append({"role": "user", "content": line})
        text = tmpl.render(history, add_generation_prompt=True)
        # a template that writes the BOS text itself must not get a second BOS id
        ids = tok.encode(text, add_special=not text.startswith(getattr(tmpl, "bos_token", "") or "\0"))
        dec = StreamDecoder(tok)
        out = []

        def on_token(seq, t):
            if t >= 0 and t not in eng.cfg.eos_ids:
                s = dec.push(t)
                out.append(s)
                sys.stdout.write(s)
                sys.stdout.flush()

        eng.add_request(ids, params, on_token=on_token)
        while eng.has_work():
            eng.step()
        sys.stdout.write(dec.flush() + "\n")
        history.append({"role": "assistant", "content": "".join(out)})
    return 0


def cmd_benchmark(args) -> int:
    """prefill tok/s, decode tok/s, TTFT p50/p99, per-run throughput (``cli/src/benchmark.rs``)."""
    import numpy as np

    from .engine.sampling_params import SamplingParams

    eng, tok, _, _ = load(args)
    rng = np.random.default_rng(args.seed)
    res = {"runs": [], "ttft_ms": []}
    for i in range(args.warmup + args.iterations):
        ids = rng.integers(0, eng.cfg.vocab, args.prompt_length).tolist()
        p = SamplingParams.greedy_params(max_tokens=args.gen_length, ignore_eos=True)
        eng.timings = {k: 0 for k in eng.timings}
        t0 = time.perf_counter()
        seqs = [eng.add_request(ids, p) for _ in range(args.batch)]
        while eng.has_work():
            eng.step()
        dt = time.perf_counter() - t0
        if i < args.warmup:
            continue
        tm = eng.timings
        res["runs"].append({"total_s": dt,
                            "prefill_tok_s": tm["prefill_tokens"] / max(tm["prefill_s"], 1e-9),
                            "decode_tok_s": tm["decode_tokens"] / max(tm["decode_s"], 1e-9),
                            "tps": (args.prompt_length + args.gen_length) * args.batch / dt})
        res["ttft_ms"] += [(s.ttft or 0) * 1e3 for s in seqs]
    tt = sorted(res["ttft_ms"])
    summary = {
        "model": os.path.basename(args.model), "batch": args.batch, "prompt_length": args.prompt_length,
        "gen_length": args.gen_length, "iterations": args.iterations,
        "prefill_tok_s": statistics.mean(r["prefill_tok_s"] for r in res["runs"]),
        "decode_tok_s": statistics.mean(r["decode_tok_s"] for r in res["runs"]),
        "tps_mean": statistics.mean(r["tps"] for r in res["runs"]),
        "tps_min": min(r["tps"] for r in res["runs"]), "tps_max": max(r["tps"] for r in res["runs"]),
        "tps_std": statistics.pstdev([r["tps"] for r in res["runs"]]),
        "ttft_p50_ms": tt[len(tt) // 2], "ttft_p99_ms": tt[min(len(tt) - 1, int(len(tt) * 0.99))],
        "rss_mb": _rss_mb(),
    }
    print(json.dumps(summary, indent=None if args.json_out else 2))
    return 0


def _rss_mb() -> float:
    try:
        with open("/proc/self/status") as f:
            for line in f:
                if line.startswith("VmRSS:"):
                    return int(line.split()[1]) / 1024.0
    except OSError:
        pass
    return 0.0


def cmd_info(args) -> int:
    """Header-only inspection: no tensor is read or dequantized."""
    from collections import Counter

    from .gguf import read_gguf_split as read_gguf
    from .models.config import config_from_gguf

    g = read_gguf(args.model)
    cfg = config_from_gguf(g.metadata, set(g.tensors))
    types = Counter(t.ggml_type.name for t in g.tensors.values())
    n_params = sum(t.n_elements for t in g.tensors.values())
    size = sum(t.nbytes for t in g.tensors.values())
    out = {"file": args.model, "gguf_version": g.version, "architecture": cfg.arch,
           "name": g.get("general.name", ""), "tensors": len(g.tensors), "parameters": n_params,
           "size_gb": round(size / 1e9, 3), "bits_per_weight": round(size * 8 / max(1, n_params), 3),
           "tensor_types": dict(types), "hparams": {k: v for k, v in cfg.to_dict().items() if k != "extra"},
           "metadata_keys": len(g.metadata)}
    print(json.dumps(out, indent=2, default=str))
    return 0


def cmd_tokenize(args) -> int:
    """Token ids and pieces of a text under the model's tokenizer (the reference's tokenizer debugging
    tool, ``cli/src/debug_tokenizer.rs``): one JSON object, or ``--ids-only`` for a comma list."""
    _, tok, tmpl, _ = load(args, need_engine=False)
    text = args.prompt
    if args.chat:
        text = tmpl.render([{"role": "user", "content": text}], add_generation_prompt=True)
    ids = tok.encode(text, add_special=not args.no_special)
    if args.ids_only:
        print(",".join(str(i) for i in ids))
        return 0
    pieces = [tok.decode([i]) for i in ids]
    print(json.dumps({"text": text, "n_tokens": len(ids), "ids": ids, "pieces": pieces,
                      "round_trip": tok.decode(ids)}, ensure_ascii=False))
    return 0


def cmd_bench_serve(args) -> int:
    """Concurrent streaming requests against a running OpenAI-compatible server; JSON summary."""
    import asyncio

    from .server.bench_serve import run

    out = asyncio.run(run(args.url, n_requests=args.requests, concurrency=args.concurrency,
                          prompt_words=args.prompt_words, max_tokens=args.max_tokens, rate=args.rate,
                          chat=args.chat, model=args.model_id, seed=args.seed, temperature=args.temperature,
                          api_key=args.api_key))
    print(json.dumps(out, indent=2))
    return 0 if out["completed"] else 1


def cmd_convert(args) -> int:
    from .gguf import QUANT_NAME_TO_TYPE
    from .models.convert import convert_gguf

    from .gguf.ikq import IKQ_NAMES, gguf_to_ikq, ikq_to_gguf

    q = args.quantize.lower()
    src = args.input
    if src.endswith(".ikq"):  # IKQ1 archive in: unpack to GGUF first
        if q == "keep":
            ikq_to_gguf(src, args.output)
            print(f"wrote {args.output}")
            return 0
        import tempfile

        tmp = tempfile.NamedTemporaryFile(suffix=".gguf", delete=False).name
        ikq_to_gguf(src, tmp)
        src = tmp
    if q == "q4_k_r4" or args.output.endswith(".ikq"):  # the reference's archive (CPU repack / ik types)
        if q not in IKQ_NAMES:
            raise SystemExit(f"IKQ archives hold {sorted(IKQ_NAMES)}, not {q}")
        gguf_to_ikq(src, args.output, q, device=args.device)
    else:
        convert_gguf(src, args.output, QUANT_NAME_TO_TYPE[q], keep_output_type=args.output_type,
                     device=args.device)
    print(f"wrote {args.output}")
    return 0


def cmd_make_random(args) -> int:
    import torch

    from .models import POLICIES, preset, random_tensors, write_gguf
    from .models.weights import QuantPolicy
    from .gguf import QUANT_NAME_TO_TYPE
    from .tokenizer.gguf_tokenizer import synthetic_tokenizer

    cfg = preset(args.arch)
    if args.layers:
        cfg.n_layers = args.layers
    pol = POLICIES.get(args.arch, QuantPolicy())
    if args.quant:
        pol = QuantPolicy(default=QUANT_NAME_TO_TYPE[args.quant], output=pol.output, attn=pol.attn, embed=pol.embed)
    dev = args.device or ("cuda" if torch.cuda.is_available() else "cpu")
    t = random_tensors(cfg, pol, seed=args.seed, device=dev)
    tok = synthetic_tokenizer(cfg.vocab)
    md = {"tokenizer.ggml.model": "llama", "tokenizer.ggml.tokens": tok.tokens,
          "tokenizer.ggml.scores": [float(x) for x in tok.scores], "tokenizer.ggml.token_type": tok.token_types}
    write_gguf(args.output, cfg, t, md)
    print(f"wrote {args.output} ({cfg.arch}, {cfg.n_layers} layers)")
    return 0


def _dp_front(args):
    """``--dp N``: N engine replicas (one process per GPU) behind the least-outstanding-work router.
    Returns (front, tokenizer, chat_template)."""
    from .parallel.dp import DataParallelEngine, GGUFEngineFactory, GGUFTPBuilder, TPReplicaFactory, default_devices

    if int(getattr(args, "pp", 1) or 1) > 1:
        raise SystemExit("--dp with --pp: replicas are single-GPU or tensor-parallel engines; drop --pp")
    tp = int(getattr(args, "tp", 1) or 1)
    _, tok, tmpl, md = load(args, need_engine=False)
    from .models.config import config_from_gguf

    cfg = config_from_gguf(md, set())
    a = {k: v for k, v in vars(args).items() if k != "fn"}
    if tp > 1:  # each replica is a tensor-parallel group on GPUs [r*tp, (r+1)*tp)
        import torch

        if not torch.cuda.is_available() or torch.cuda.device_count() < args.dp * tp:
            raise SystemExit(f"--dp {args.dp} --tp {tp} needs {args.dp * tp} GPUs")
        devices = [f"cuda:{r * tp}" for r in range(args.dp)]
        factory = TPReplicaFactory(GGUFTPBuilder(a), tp)
    else:
        devices = ["cpu"] * args.dp if getattr(args, "device", None) == "cpu" else default_devices(args.dp)
        factory = GGUFEngineFactory(a)
    front = DataParallelEngine(factory, devices, cfg=cfg, tokenizer=tok)
    log.info("data parallel: %d replicas on %s", front.n_alive, ", ".join(devices))
    return front, tok, tmpl


def _lockstep(eng, args):
    """Multi-rank engines (--tp / --pp under torchrun): rank 0 serves through a LockstepLeader, the
    other ranks replay its steps and return None here once it stops."""
    if int(getattr(args, "tp", 1) or 1) <= 1 and int(getattr(args, "pp", 1) or 1) <= 1:
        return eng
    import torch.distributed as dist
    from torch.distributed.distributed_c10d import _get_default_store

    from .parallel.lockstep import LockstepLeader, follower_loop

    store = _get_default_store()
    if dist.get_rank() != 0:
        follower_loop(eng, store)
        return None
    lead = LockstepLeader(eng, store)
    import atexit

    atexit.register(lead.stop)
    return lead


def cmd_server(args) -> int:
    from .server.async_engine import AsyncEngine
    from .server.uds import UDSServer

    path = args.socket or f"/tmp/barq-inference-{args.port}.sock"
    if int(getattr(args, "dp", 1) or 1) > 1:
        front, tok, tmpl = _dp_front(args)
        srv = UDSServer(front, tok, path, chat_template=tmpl)
    else:
        eng, tok, tmpl, _ = load(args)
        eng = _lockstep(eng, args)
        if eng is None:  # a follower rank: rank 0 has stopped serving
            return 0
        srv = UDSServer(AsyncEngine(eng), tok, path, chat_template=tmpl)
    if getattr(args, "metrics_port", 0):
        from .server.metrics import InferenceMetrics
        from .server.metrics_server import MetricsServer, MetricsServerConfig

        srv.metrics = InferenceMetrics()
        ms = MetricsServer(srv.metrics, MetricsServerConfig(port=args.metrics_port),
                           health_fn=lambda: (srv.ae.healthy, srv.ae.last_error)).start()
        print(f"barq metrics on :{ms.port} (/metrics, /metrics.json, /health)")
    print(f"barq UDS server listening on {path}")
    srv.start(background=False)
    return 0


def _serve_native_front_end(aengine, tok, tmpl, args) -> int:
    """HTTP served by the C++ front end ``barq-http``: the engine answers on a private UDS socket."""
    import subprocess
    import tempfile

    from .server.uds import UDSServer
    from .server.uds_native import build_http

    exe = build_http()
    sock = os.path.join(tempfile.mkdtemp(prefix="barq-"), "engine.sock")
    srv = UDSServer(aengine, tok, sock, chat_template=tmpl).start()
    cmd = [exe, "--socket", sock, "--host", args.host, "--port", str(args.port),
           "--model-id", os.path.basename(args.model), "--rpm", str(max(0, args.rate_limit_rpm))]
    env = dict(os.environ)
    if getattr(args, "api_key", None):
        env["BARQ_API_KEY"] = args.api_key  # through the environment, not the command line
    try:
        return subprocess.call(cmd, env=env)
    except KeyboardInterrupt:
        return 0
    finally:
        srv.stop()


_DROP_WITH_VALUE = ("--dp", "--host", "--port", "--rate-limit-rpm", "--socket", "--api-key")


def _engine_server_argv(argv: list[str]) -> list[str]:
    """The command line of one engine process for ``http-server --native-front-end --dp N``: this
    process's arguments with ``http-server`` turned into ``server`` and the front-end options
    (--dp, --host, --port, --rate-limit-rpm, --api-key, --native-front-end) removed."""
    out, i = [], 0
    while i < len(argv):
        a = argv[i]
        if a == "http-server":
            out.append("server")
        elif a == "--native-front-end":
            pass
        elif a in _DROP_WITH_VALUE:
            i += 1  # and its value
        elif any(a.startswith(f + "=") for f in _DROP_WITH_VALUE):
            pass
        else:
            out.append(a)
        i += 1
    return out


def _serve_native_replicas(args) -> int:
    """``http-server --native-front-end --dp N``: N engine processes, each a UDS server on its own
    GPU (``CUDA_VISIBLE_DEVICES``), behind one ``barq-http`` that balances them -- data parallelism
    with no Python router in the request path."""
    import socket as _socket
    import subprocess
    import tempfile

    from .server.uds_native import build_http

    n = int(args.dp)
    exe = build_http()
    tmp = tempfile.mkdtemp(prefix="barq-dp-")
    socks = [os.path.join(tmp, f"engine{i}.sock") for i in range(n)]
    base = _engine_server_argv(list(getattr(args, "_argv", sys.argv[1:])))
    device = getattr(args, "device", None) or ("cuda" if _cuda() else "cpu")
    visible = os.environ.get("CUDA_VISIBLE_DEVICES")
    devs = [d for d in visible.split(",") if d.strip()] if visible else [str(i) for i in range(n)]
    procs = []
    try:
        for i, sock in enumerate(socks):
            env = dict(os.environ)
            if device != "cpu":
                env["CUDA_VISIBLE_DEVICES"] = devs[i % len(devs)]
            procs.append(subprocess.Popen([sys.executable, "-m", "barq_inference_b200.cli", *base, "--socket", sock],
                                          env=env))
        deadline = time.monotonic() + float(os.environ.get("BARQ_ENGINE_START_TIMEOUT", "3600"))
        pending = set(range(n))
        while pending:  # an engine is ready once its UDS server accepts connections
            for i in list(pending):
                if procs[i].poll() is not None:
                    raise RuntimeError(f"engine {i} exited with code {procs[i].returncode} before serving")
                try:
                    with _socket.socket(_socket.AF_UNIX, _socket.SOCK_STREAM) as c:
                        c.connect(socks[i])
                    pending.discard(i)
                except OSError:
                    pass
            if time.monotonic() > deadline:
                raise TimeoutError(f"engines {sorted(pending)} not serving in time")
            time.sleep(0.2)
        cmd = [exe, "--host", args.host, "--port", str(args.port), "--model-id", os.path.basename(args.model),
               "--rpm", str(max(0, args.rate_limit_rpm))]
        for sock in socks:
            cmd += ["--socket", sock]
        import signal

        # a SIGTERM to this process alone still stops the front end and every engine (finally below)
        signal.signal(signal.SIGTERM, lambda *_: sys.exit(0))
        fenv = dict(os.environ)
        if getattr(args, "api_key", None):
            fenv["BARQ_API_KEY"] = args.api_key  # through the environment, not the command line
        front = subprocess.Popen(cmd, env=fenv)
        procs.insert(0, front)  # stopped first: it drains, then the engines go
        try:
            return front.wait()
        except KeyboardInterrupt:
            return 0
    finally:
        # the front end first (it drains its requests in flight), then every engine
        for group in (procs[:1], procs[1:]) if len(procs) > n else ((), procs):
            for pr in group:
                if pr.poll() is None:
                    pr.terminate()
            for pr in group:
                try:
                    pr.wait(timeout=40)
                except subprocess.TimeoutExpired:
                    pr.kill()


def cmd_http_server(args) -> int:
    from .server.async_engine import AsyncEngine
    from .server.openai_api import OpenAIServer, serve

    native = bool(getattr(args, "native_front_end", False))
    if native and int(getattr(args, "dp", 1) or 1) > 1 and int(getattr(args, "tp", 1) or 1) == 1:
        return _serve_native_replicas(args)
    if int(getattr(args, "dp", 1) or 1) > 1:
        front, tok, tmpl = _dp_front(args)
        if native:
            return _serve_native_front_end(front, tok, tmpl, args)
        srv = OpenAIServer(front, tok, model_id=os.path.basename(args.model), chat_template=tmpl,
                           rate_limit_rpm=args.rate_limit_rpm, arch=front.cfg.arch, aengine=front,
                           api_key=args.api_key)
    else:
        eng, tok, tmpl, md = load(args)
        eng = _lockstep(eng, args)
        if eng is None:  # a follower rank: rank 0 has stopped serving
            return 0
        if native:
            return _serve_native_front_end(AsyncEngine(eng), tok, tmpl, args)
        srv = OpenAIServer(eng, tok, model_id=os.path.basename(args.model), chat_template=tmpl,
                           rate_limit_rpm=args.rate_limit_rpm, arch=eng.cfg.arch, api_key=args.api_key)
    serve(srv, args.host, args.port)
    return 0


def cmd_metal_info(args) -> int:
    print(json.dumps({"metal": "unavailable", "reason": "Apple Metal is not part of this B200 (CUDA) build"}))
    return 0


def cmd_wasm_info(args) -> int:
    print(json.dumps({"wasm": "informational only", "webgpu": False, "wasm_simd": False,
                      "recommended_quant": "q4_0 for browser heaps <= 4 GB"}))
    return 0


def cmd_device_info(args) -> int:
    import torch

    d = {"cuda": torch.cuda.is_available()}
    if d["cuda"]:
        p = torch.cuda.get_device_properties(0)
        d.update(name=p.name, sm_count=p.multi_processor_count, memory_gb=round(p.total_memory / 1e9, 1),
                 capability=f"{p.major}.{p.minor}", devices=torch.cuda.device_count())
    print(json.dumps(d))
    return 0


# ------------------------------------------------------------------ parser
def build_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(prog="barq", description="Blackwell-native GGUF inference engine")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("-t", "--threads", type=int, default=4)
    ap.add_argument("--cuda-graphs", dest="cuda_graphs", action="store_true", default=None)
    ap.add_argument("--no-cuda-graphs", dest="cuda_graphs", action="store_false")
    ap.add_argument("--flash-attn", action="store_true", help="always on (paged flash attention kernels)")
    ap.add_argument("--log-format", choices=["text", "json"], default="text",
                    help="json: one structured object per line with request ids (production logging)")
    ap.add_argument("--log-file", default=None)
    ap.add_argument("--preset", choices=["max-speed", "balanced", "max-quality", "cpu", "gpu"])
    sub = ap.add_subparsers(dest="cmd", required=True)

    def model_args(p):
        p.add_argument("-m", "--model", required=True)
        p.add_argument("--device", choices=["cuda", "cpu"])
        p.add_argument("--context-size", type=int, default=2048)
        p.add_argument("--kv-dtype", choices=["fp16", "bf16", "fp8"], default="fp16")
        p.add_argument("--kv-cache-gb", type=float, default=8.0)
        p.add_argument("--max-batch", type=int, default=64)
        p.add_argument("--tp", type=int, default=1, help="tensor-parallel ranks (launch with torchrun)")
        p.add_argument("--ep", type=int, default=0,
                       help="expert-parallel ranks (experts are split over the --tp ranks; must equal --tp)")
        p.add_argument("--pp", type=int, default=1, help="pipeline stages (launch with torchrun; layers split contiguously)")
        p.add_argument("--dp", type=int, default=1,
                       help="data-parallel replicas for server/http-server: one engine process per GPU behind a "
                            "least-outstanding-work request router")
        p.add_argument("--comm", choices=["fused", "nccl"], default="fused",
                       help="TP all-reduce: fused one-shot kernel over NVLink peer memory, or NCCL")
        p.add_argument("--block-size", type=int, default=16, help="KV cache page size (tokens)")
        p.add_argument("--no-fmoe", action="store_true", help="unfused per-expert MoE loop (baseline)")
        p.add_argument("--prefix-cache", action="store_true")
        p.add_argument("--max-waiting", type=int, default=0,
                       help="admission control: refuse requests (HTTP 503) beyond this many waiting (0: no limit)")
        p.add_argument("--mla", action="store_true", help="DeepSeek MLA latent cache (on for deepseek2 models)")
        p.add_argument("--fmoe", action="store_true", help="fused MoE routing/dispatch (default path)")
        p.add_argument("--ser", action="store_true", help="smart expert reduction: drop experts with gate < 0.2")

    def sampling_args(p):
        p.add_argument("--max-tokens", type=int, default=128)
        p.add_argument("--temperature", type=float, default=0.8)
        p.add_argument("--top-k", type=int, default=40)
        p.add_argument("--top-p", type=float, default=0.95)
        p.add_argument("--min-p", type=float, default=0.0)
        p.add_argument("--repeat-penalty", type=float, default=1.0)
        p.add_argument("--seed", type=int, default=0)

    p = sub.add_parser("run", help="generate from a prompt")
    model_args(p)
    sampling_args(p)
    p.add_argument("-p", "--prompt", default="Hello")
    p.add_argument("--prompt-ids", default="", help="comma-separated token ids (bypasses the tokenizer)")
    p.add_argument("--prompt-cache", default=None,
                   help="KV session file: reused when present (prompt prefix skips prefill), written after the run")
    p.add_argument("--chat-format", action="store_true")
    p.add_argument("--json", action="store_true", help="constrain output to JSON")
    p.add_argument("--speculative", action="store_true")
    p.add_argument("--draft-model")
    p.add_argument("--draft-max", type=int, default=16)
    p.add_argument("--lookup-decoding", action="store_true",
                   help="speculative decoding with drafts copied from earlier n-grams of the context (no draft model)")
    p.add_argument("--lookup-ngram", type=int, default=3, help="longest n-gram matched by --lookup-decoding")
    p.add_argument("--speculation-preset", choices=["default", "code", "creative", "max_speed"], default="default")
    p.set_defaults(fn=cmd_run)

    p = sub.add_parser("chat", help="interactive chat")
    model_args(p)
    sampling_args(p)
    p.add_argument("--system-prompt", default="")
    p.set_defaults(fn=cmd_chat)

    p = sub.add_parser("benchmark", help="prefill/decode throughput and TTFT")
    model_args(p)
    p.add_argument("--iterations", type=int, default=10)
    p.add_argument("--warmup", type=int, default=2)
    p.add_argument("--prompt-length", type=int, default=512)
    p.add_argument("--gen-length", type=int, default=128)
    p.add_argument("--batch", type=int, default=1)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--json-out", action="store_true")
    p.set_defaults(fn=cmd_benchmark)

    p = sub.add_parser("info", help="print GGUF header, hparams and tensor types")
    p.add_argument("-m", "--model", required=True)
    p.set_defaults(fn=cmd_info)

    p = sub.add_parser("tokenize", help="token ids and pieces of a text under the model's tokenizer")
    p.add_argument("-m", "--model", required=True)
    p.add_argument("-p", "--prompt", required=True)
    p.add_argument("--chat", action="store_true", help="render the text as a user turn of the chat template first")
    p.add_argument("--no-special", action="store_true", help="no BOS / special tokens")
    p.add_argument("--ids-only", action="store_true")
    p.set_defaults(fn=cmd_tokenize)

    p = sub.add_parser("bench-serve", help="load-test a running OpenAI-compatible server (TTFT, ITL, throughput)")
    p.add_argument("--url", default="http://127.0.0.1:8000")
    p.add_argument("--requests", type=int, default=64)
    p.add_argument("--concurrency", type=int, default=16)
    p.add_argument("--rate", type=float, default=0.0, help="Poisson arrivals per second (0: all at once)")
    p.add_argument("--prompt-words", type=int, default=64)
    p.add_argument("--max-tokens", type=int, default=128)
    p.add_argument("--temperature", type=float, default=0.0)
    p.add_argument("--chat", action="store_true", help="use /v1/chat/completions")
    p.add_argument("--model-id", default="barq")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--api-key", default=os.environ.get("BARQ_API_KEY"), help="sent as 'Authorization: Bearer KEY'")
    p.set_defaults(fn=cmd_bench_serve)

    p = sub.add_parser("convert", help="requantize a GGUF file")
    p.add_argument("--input", required=True)
    p.add_argument("--output", required=True)
    p.add_argument("--quantize", default="q4_k",
                   help="ggml type (q4_k, q6_k, ..., iq4_ks, iq3_ks, iq2_ks), q4_k_r4 (IKQ archive) or keep")
    p.add_argument("--output-type", default=None, help="type for output.weight (default: keep)")
    p.add_argument("--device", default=None)
    p.set_defaults(fn=cmd_convert)

    p = sub.add_parser("make-random-gguf", help="write a random-init checkpoint of a preset architecture")
    p.add_argument("--arch", default="tiny")
    p.add_argument("--output", required=True)
    p.add_argument("--quant", default=None)
    p.add_argument("--layers", type=int, default=0)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--device", default=None)
    p.set_defaults(fn=cmd_make_random)

    p = sub.add_parser("server", help="Unix-domain-socket streaming server")
    model_args(p)
    p.add_argument("--host", default="127.0.0.1")
    p.add_argument("--port", type=int, default=8080)
    p.add_argument("--socket", default=None)
    p.add_argument("--metrics-port", type=int, default=0, help="serve /metrics and /health on this port (e.g. 9090; 0: off)")
    p.set_defaults(fn=cmd_server)

    p = sub.add_parser("http-server", help="OpenAI-compatible HTTP server")
    model_args(p)
    p.add_argument("--host", default="0.0.0.0")
    p.add_argument("--port", type=int, default=8000)
    p.add_argument("--rate-limit-rpm", type=int, default=60)
    p.add_argument("--api-key", default=os.environ.get("BARQ_API_KEY"),
                   help="require 'Authorization: Bearer KEY' on the /v1 routes (default: $BARQ_API_KEY)")
    p.add_argument("--native-front-end", action="store_true",
                   help="serve HTTP from the C++ front end barq-http (engine behind a private UDS socket)")
    p.set_defaults(fn=cmd_http_server)

    sub.add_parser("metal-info").set_defaults(fn=cmd_metal_info)
    sub.add_parser("wasm-info").set_defaults(fn=cmd_wasm_info)
    sub.add_parser("device-info").set_defaults(fn=cmd_device_info)
    return ap


def main(argv=None) -> int:
    args = build_parser().parse_args(argv)
    args._argv = list(argv) if argv is not None else sys.argv[1:]  # for commands that start children
    logging.basicConfig(level=logging.DEBUG if args.verbose else logging.INFO, format="%(message)s")
    if args.log_format == "json" or args.log_file:
        from .utils.logging import LoggingConfig, init_logger

        init_logger(LoggingConfig(min_level=logging.DEBUG if args.verbose else logging.INFO,
                                  json_format=args.log_format == "json", log_file=args.log_file))
    try:
        import torch

        torch.set_num_threads(max(1, args.threads))
    except Exception:
        pass
    return int(args.fn(args) or 0)


if __name__ == "__main__":
    sys.exit(main())
