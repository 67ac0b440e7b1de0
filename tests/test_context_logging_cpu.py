"""ContextParams presets -> engine switches; structured JSON logging with request ids (CPU)."""
import json
import logging

from barq_inference_b200.engine.context_params import ContextParams
from barq_inference_b200.models import POLICIES, preset, random_tensors
from barq_inference_b200.utils.logging import LoggingConfig, init_logger, request_logger


def test_context_params_map_to_engine_config():
    ec = ContextParams.gpu_optimized().engine_config(model_max_ctx=4096)
    assert ec.max_model_len == 4096 and ec.max_num_seqs == 64 and ec.max_num_batched_tokens == 8192
    assert ec.kv_dtype == "fp16"
    assert ContextParams.speed().engine_config().kv_dtype == "fp8"
    assert ContextParams.speed().engine_config().max_model_len == 4096
    assert ContextParams.quality().kv_dtype() == "bf16"
    assert ContextParams(type_k=1, type_v=8).kv_dtype() == "fp8"  # the narrower of K and V wins
    cp = ContextParams(n_batch=2048, n_ubatch=256, n_seq_max=8)
    ec = cp.engine_config(model_max_ctx=512, device="cpu")
    assert ec.max_num_batched_tokens == 256 and ec.max_num_seqs == 8 and ec.max_model_len == 512
    assert ec.device == "cpu"


def test_context_params_model_overrides_and_cpu_engine():
    cfg = preset("tiny", n_layers=1, vocab=300, max_ctx=256)
    cp = ContextParams(n_ctx=128, rope_freq_base=20000.0, rope_freq_scale=0.5, n_gpu_layers=0, n_threads=2)
    m = cp.apply_to_model(cfg)
    assert m.rope_theta == 20000.0 and m.rope_scaling == "linear" and m.rope_factor == 2.0 and m.max_ctx == 128
    eng = cp.make_engine(cfg, random_tensors(cfg, POLICIES["tiny"], seed=0))
    assert type(eng).__name__ == "CPUEngine" and eng.max_model_len == 128
    assert not ContextParams.cpu_optimized().use_gpu


def test_json_logging_with_request_ids(tmp_path):
    path = tmp_path / "log.jsonl"
    init_logger(LoggingConfig.production(log_file=str(path)))
    try:
        logging.getLogger("barq.engine").info("engine up %d", 3)
        request_logger("req-42").warning("slow", extra={"context": {"latency_ms": 12.5}})
        logging.getLogger("barq.engine").debug("hidden")  # below INFO
    finally:
        init_logger(LoggingConfig(log_to_stdout=False))  # detach the file handler
    lines = [json.loads(x) for x in path.read_text().splitlines()]
    assert [x["message"] for x in lines] == ["engine up 3", "slow"]
    assert lines[0]["level"] == "INFO" and lines[0]["module"] == "barq.engine" and "request_id" not in lines[0]
    assert lines[1]["level"] == "WARN" and lines[1]["request_id"] == "req-42"
    assert lines[1]["context"] == {"latency_ms": 12.5} and isinstance(lines[1]["timestamp"], int)


def test_http_request_log_line(tmp_path):
    from fastapi.testclient import TestClient

    from barq_inference_b200.engine.cpu_engine import CPUEngine
    from barq_inference_b200.server.openai_api import OpenAIServer
    from barq_inference_b200.tokenizer.gguf_tokenizer import synthetic_tokenizer

    cfg = preset("tiny", n_layers=1, vocab=600, max_ctx=256)
    eng = CPUEngine(cfg, random_tensors(cfg, POLICIES["tiny"], seed=0), max_model_len=256)
    srv = OpenAIServer(eng, synthetic_tokenizer(cfg.vocab))
    path = tmp_path / "http.jsonl"
    init_logger(LoggingConfig(log_to_stdout=False, log_file=str(path)))
    try:
        r = TestClient(srv.app).post("/v1/completions", json={"prompt": "hi", "max_tokens": 2},
                                     headers={"x-request-id": "abc123"})
        assert r.status_code == 200 and r.headers["x-request-id"] == "abc123"
    finally:
        init_logger(LoggingConfig(log_to_stdout=False))
        srv.aengine.shutdown()
    rec = [json.loads(x) for x in path.read_text().splitlines()]
    assert any(x.get("request_id") == "abc123" and x["context"]["status"] == 200 for x in rec), rec
