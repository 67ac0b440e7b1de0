"""Expert-load counting and balance measures (reference aux loss) on the fp32 MoE forward (CPU)."""
import torch

from barq_inference_b200.models import POLICIES, preset, random_tensors
from barq_inference_b200.models.moe_stats import ExpertLoad, enable
from barq_inference_b200.models.reference import ReferenceModel


def test_counts_from_routing_and_aux_loss():
    cfg = preset("tiny-moe")
    m = ReferenceModel(cfg, random_tensors(cfg, POLICIES["tiny"], seed=0))
    load = enable(m)
    m.forward(list(range(1, 21)))
    s = load.summary(aux_loss_coef=0.5)
    n_moe = sum(cfg.layer_is_moe(i) for i in range(cfg.n_layers))
    assert s["tokens_routed"] == 20 * cfg.n_experts_used * n_moe
    c = torch.tensor(s["per_layer"], dtype=torch.float64)
    want = (0.5 * ((c - c.mean(1, keepdim=True)) ** 2).mean(1)).mean().item()
    assert abs(s["aux_loss"] - want) < 1e-9 and s["max_over_mean"] >= 1.0


def test_even_load_has_zero_loss():
    load = ExpertLoad(2, 4)
    load.add(0, torch.tensor([5, 5, 5, 5]))
    s = load.summary()
    assert s["aux_loss"] == 0.0 and s["max_over_mean"] == 1.0 and s["cv"] == 0.0 and s["tokens_routed"] == 20
    load.reset()
    assert load.summary()["tokens_routed"] == 0


def test_prometheus_exposes_expert_load():
    from barq_inference_b200.engine.cpu_engine import CPUEngine
    from barq_inference_b200.engine.sampling_params import SamplingParams
    from barq_inference_b200.server.metrics import InferenceMetrics

    cfg = preset("tiny-moe")
    eng = CPUEngine(cfg, random_tensors(cfg, POLICIES["tiny"], seed=0), max_model_len=256)
    enable(eng.model)
    eng.generate([[1, 2, 3, 4]], SamplingParams.greedy_params(max_tokens=3))
    text = InferenceMetrics().prometheus(eng)
    assert "barq_moe_tokens_routed_total" in text and "barq_moe_load_max_over_mean" in text
