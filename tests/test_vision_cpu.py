"""Vision scaffolding: image ops, the deterministic patch encoder, multimodal prompts (CPU)."""
import numpy as np
import pytest
import torch

from barq_inference_b200.models import POLICIES, preset, random_tensors
from barq_inference_b200.models.vision import (ClipVisionEncoder, ImageInput, ImagePreprocessor, LlavaModel,
                                               Qwen2VlModel, fuse_text_and_image_embeddings, insert_image_tokens)


def test_image_resize_and_normalize():
    img = ImageInput.solid_rgb(2, 2, [255, 0, 0])
    r = img.resize_nearest(4, 4)
    assert (r.width, r.height) == (4, 4)
    n = r.normalize()
    assert n.shape == (48,) and n[0] == 1.0 and n[1] == 0.0
    with pytest.raises(ValueError):
        ImageInput.new(2, 2, b"\0" * 11)
    with pytest.raises(ValueError):
        img.resize_nearest(0, 3)
    grad = ImageInput.new(2, 1, [0, 0, 0, 200, 100, 50])
    assert grad.resize_nearest(4, 1).pixels == bytes([0, 0, 0] * 2 + [200, 100, 50] * 2)
    assert ImagePreprocessor(1, 1, False).preprocess(grad).tolist() == [0.0, 0.0, 0.0]


def _encode_loop(enc, img):
    """The patch-mean + position formula written as plain loops."""
    w, h = enc.image_size()
    p, D = enc.patch_size(), enc.embedding_dim()
    px = enc.preprocess(img).reshape(h, w, 3)
    nx, ny = w // p, h // p
    out = np.zeros((nx * ny, D), np.float32)
    for py in range(ny):
        for qx in range(nx):
            i = py * nx + qx
            m = px[py * p:(py + 1) * p, qx * p:(qx + 1) * p].reshape(-1, 3).mean(0)
            for d in range(D):
                out[i, d] = m[d % 3] + i / (nx * ny) + d / D * 0.1
    return out


def test_clip_encoder_shapes_and_values():
    enc = ClipVisionEncoder((4, 4), 2, 8)
    e = enc.encode(ImageInput.solid_rgb(2, 2, [64, 128, 255]))
    assert tuple(e.shape) == (4, 8)
    rng = np.random.default_rng(0)
    img = ImageInput.new(12, 8, rng.integers(0, 256, 12 * 8 * 3, dtype=np.uint8))
    enc = ClipVisionEncoder((8, 6), 2, 10)
    assert np.allclose(enc.encode(img).numpy(), _encode_loop(enc, img), atol=1e-5)


def test_prompt_helpers():
    assert insert_image_tokens("answer this ", 2) == "answer this <image> <image>"
    assert insert_image_tokens("x", 0) == "x"
    f = fuse_text_and_image_embeddings(torch.ones(2, 4), torch.zeros(3, 4))
    assert tuple(f.shape) == (5, 4)
    with pytest.raises(ValueError):
        fuse_text_and_image_embeddings(torch.ones(2, 4), torch.zeros(3, 5))


def test_multimodal_prompt_on_cpu_engine():
    """Image rows replace the placeholder embeddings: the output differs from the text-only run
    with the same placeholder ids, and equals a reference forward given the same embeddings."""
    from barq_inference_b200.engine.cpu_engine import CPUEngine
    from barq_inference_b200.engine.sampling_params import SamplingParams
    from barq_inference_b200.models.reference import ReferenceModel

    cfg = preset("tiny")
    tensors = random_tensors(cfg, POLICIES["tiny"], seed=0)
    eng = CPUEngine(cfg, tensors, max_model_len=512)
    with pytest.raises(ValueError):
        Qwen2VlModel(eng)  # tiny preset is a llama arch
    vlm = LlavaModel(eng)
    img = ImageInput.solid_rgb(224, 224, [10, 200, 30])
    e = vlm.image_embeddings(img)
    assert tuple(e.shape) == (196, cfg.hidden)
    prompt = [5, 6, 7]
    res = vlm.generate(prompt, img, SamplingParams.greedy_params(max_tokens=4))
    ids = prompt + [0] * 196
    ref = ReferenceModel(cfg, tensors)
    lg = ref.forward(ids, {}, embeds=(3, e))[-1]
    assert res.tokens[0] == int(lg.argmax())
    lg_text = ref.forward(ids, {})[-1]
    assert not torch.allclose(lg, lg_text)
