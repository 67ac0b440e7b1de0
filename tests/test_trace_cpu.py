"""BARQ_PROFILE step records on the CPU engine path (no GPU)."""
import json

from barq_inference_b200.utils.trace import StepProfiler, nvtx


class _Plan:
    kind = "decode"
    n_new = [1, 1, 1]


class _Eng:
    def __init__(self):
        import torch

        self.device = torch.device("cpu")
        self.step_count = 0
        self.last_plan = _Plan()


def test_step_profiler_writes_json(tmp_path, monkeypatch):
    out = tmp_path / "prof.jsonl"
    monkeypatch.setenv("BARQ_PROFILE", "1")
    monkeypatch.setenv("BARQ_PROFILE_FILE", str(out))
    eng = _Eng()
    prof = StepProfiler.from_env(eng)
    for i in range(3):
        eng.step_count = i
        prof.step(lambda: [])
    prof.flush()
    recs = [json.loads(x) for x in out.read_text().splitlines()]
    assert [r["step"] for r in recs] == [0, 1, 2]
    assert all(r["kind"] == "decode" and r["tokens"] == 3 and r["wall_ms"] >= 0 for r in recs)


def test_profiler_off_by_default(monkeypatch):
    monkeypatch.delenv("BARQ_PROFILE", raising=False)
    monkeypatch.delenv("BARQ_NVTX", raising=False)
    assert StepProfiler.from_env(_Eng()) is None
    with nvtx("noop"):  # no CUDA needed when disabled
        pass
