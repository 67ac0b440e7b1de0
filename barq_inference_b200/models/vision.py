"""Vision scaffolding for multimodal models: image input, preprocessing, a deterministic patch
encoder, a projector into the language model's embedding space and the LLaVA / Qwen2-VL wrappers.

Parity: ``models/src/vision/mod.rs`` (``ImageInput``, ``ImagePreprocessor``, ``VisionEncoder``,
``ClipVisionEncoder``), ``models/src/llava.rs:27-100`` and ``models/src/qwen2vl.rs:27-100``.

The reference's encoder is a placeholder: per patch, the mean of each RGB channel, mixed into
every embedding dimension (``dim % 3`` picks the channel) plus a position term
``patch / n_patches + 0.1 * dim / embedding_dim``.  The same function is computed here with
tensor ops (an average pool over the patch grid), on whatever device the image is sent to.
Beyond the reference, :class:`VisionLanguageModel` actually runs a multimodal prompt: the patch
embeddings go through a linear projector (from ``mm.*`` tensors when a checkpoint has them,
otherwise a seeded random init) and replace the input embeddings of the image placeholder
positions of the prompt (``Engine.add_request(embeds=...)``), so the language model attends to
them like to any other prompt rows.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch
import torch.nn.functional as F

IMAGE_TOKEN = "<image>"


@dataclass(frozen=True)
class ImageInput:
    """Raw RGB image, ``pixels`` = height x width x 3 bytes, row-major."""

    width: int
    height: int
    pixels: bytes

    @staticmethod
    def new(width: int, height: int, pixels) -> "ImageInput":
        px = bytes(pixels)
        if width < 0 or height < 0 or len(px) != width * height * 3:
            raise ValueError(f"expected {width * height * 3} RGB bytes, got {len(px)}")
        return ImageInput(width, height, px)

    @staticmethod
    def solid_rgb(width: int, height: int, rgb) -> "ImageInput":
        return ImageInput(width, height, bytes(rgb) * (width * height))

    def array(self) -> np.ndarray:
        return np.frombuffer(self.pixels, np.uint8).reshape(self.height, self.width, 3)

    def resize_nearest(self, width: int, height: int) -> "ImageInput":
        if width <= 0 or height <= 0:
            raise ValueError("image dimensions must be non-zero")
        if (width, height) == (self.width, self.height):
            return self
        ys = np.arange(height) * self.height // height
        xs = np.arange(width) * self.width // width
        return ImageInput(width, height, self.array()[ys][:, xs].tobytes())

    def normalize(self) -> np.ndarray:
        """Bytes / 255 as float32, same order as ``pixels``."""
        return np.frombuffer(self.pixels, np.uint8).astype(np.float32) / 255.0


@dataclass(frozen=True)
class ImagePreprocessor:
    target_width: int
    target_height: int
    normalize: bool = True

    def preprocess(self, image: ImageInput) -> np.ndarray:
        r = image.resize_nearest(self.target_width, self.target_height)
        return r.normalize() if self.normalize else np.frombuffer(r.pixels, np.uint8).astype(np.float32)


class VisionEncoder:
    """Interface: image -> [n_patches, embedding_dim] patch embeddings."""

    def image_size(self) -> tuple[int, int]:
        raise NotImplementedError

    def patch_size(self) -> int:
        raise NotImplementedError

    def embedding_dim(self) -> int:
        raise NotImplementedError

    def preprocess(self, image: ImageInput) -> np.ndarray:
        raise NotImplementedError

    def encode(self, image: ImageInput, device=None) -> torch.Tensor:
        raise NotImplementedError


class ClipVisionEncoder(VisionEncoder):
    def __init__(self, image_size: tuple[int, int] = (224, 224), patch_size: int = 16, embedding_dim: int = 768):
        self.pre = ImagePreprocessor(image_size[0], image_size[1], True)
        self._patch = patch_size
        self._dim = embedding_dim

    def image_size(self) -> tuple[int, int]:
        return self.pre.target_width, self.pre.target_height

    def patch_size(self) -> int:
        return self._patch

    def embedding_dim(self) -> int:
        return self._dim

    def n_patches(self) -> int:
        return (self.pre.target_width // self._patch) * (self.pre.target_height // self._patch)

    def preprocess(self, image: ImageInput) -> np.ndarray:
        return self.pre.preprocess(image)

    def encode(self, image: ImageInput, device=None) -> torch.Tensor:
        w, h = self.image_size()
        p = self._patch
        px = torch.from_numpy(self.preprocess(image).copy()).to(device).view(h, w, 3)
        px = px[: h // p * p, : w // p * p].permute(2, 0, 1)[None]  # [1, 3, H, W]
        means = F.avg_pool2d(px, p)[0].flatten(1).T  # [n_patches, 3], row-major patch order
        n, D = means.shape[0], self._dim
        dims = torch.arange(D, device=px.device)
        mix = means[:, dims % 3]  # [n, D]
        pos = torch.arange(n, device=px.device, dtype=torch.float32)[:, None] / max(n, 1) + \
            (dims.float() / max(D, 1) * 0.1)[None]
        return mix + pos


class Projector:
    """Linear map (with optional GELU-MLP second layer) from patch embeddings to the LM hidden size.

    Weights come from ``mm.0.weight`` / ``mm.0.bias`` (and ``mm.2.*``), the tensor names of
    llama.cpp's multimodal projector files, when given; otherwise a seeded random init."""

    def __init__(self, in_dim: int, hidden: int, tensors: dict | None = None, seed: int = 0, device=None):
        self.layers = []
        if tensors and "mm.0.weight" in tensors:
            for i in (0, 2):
                if f"mm.{i}.weight" in tensors:
                    w = torch.as_tensor(tensors[f"mm.{i}.weight"], dtype=torch.float32)
                    b = tensors.get(f"mm.{i}.bias")
                    b = torch.as_tensor(b, dtype=torch.float32) if b is not None else torch.zeros(w.shape[0])
                    self.layers.append((w.to(device), b.to(device)))
        else:
            g = torch.Generator().manual_seed(seed)
            w = torch.randn(hidden, in_dim, generator=g) / in_dim ** 0.5
            self.layers.append((w.to(device), torch.zeros(hidden, device=device)))
        if self.layers[-1][0].shape[0] != hidden or self.layers[0][0].shape[1] != in_dim:
            raise ValueError("projector: weight shapes do not match the encoder / model sizes")

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        for i, (w, b) in enumerate(self.layers):
            if i:
                x = F.gelu(x)
            x = x.to(w.device) @ w.T + b
        return x


def insert_image_tokens(prompt: str, images: int) -> str:
    """``prompt`` followed by ``images`` space-separated ``<image>`` markers."""
    if images == 0:
        return prompt
    return prompt.rstrip() + " " + " ".join([IMAGE_TOKEN] * images)


def fuse_text_and_image_embeddings(text: torch.Tensor, image: torch.Tensor) -> torch.Tensor:
    """Concatenate [n_text, D] and [n_image, D] along the sequence axis."""
    if text.dim() != 2 or image.dim() != 2:
        raise ValueError("expected rank-2 embeddings")
    if text.shape[1] != image.shape[1]:
        raise ValueError("embedding dimensions must match")
    return torch.cat([text, image.to(text.device, text.dtype)], 0)


class VisionLanguageModel:
    """A language model (``Engine`` or ``CPUEngine``) plus an image encoder and projector."""

    ARCHES: tuple[str, ...] = ()
    ENCODER = dict(image_size=(224, 224), patch_size=16, embedding_dim=768)

    def __init__(self, engine, projector_tensors: dict | None = None, strict_arch: bool = True):
        arch = engine.cfg.arch
        if strict_arch and self.ARCHES and arch not in self.ARCHES:
            raise ValueError(f"expected {' / '.join(self.ARCHES)} architecture, got {arch}")
        self.engine = engine
        self.encoder = ClipVisionEncoder(**self.ENCODER)
        dev = getattr(engine, "device", None)
        self.projector = Projector(self.encoder.embedding_dim(), engine.cfg.hidden, projector_tensors, device=dev)

    def vision_encoder(self) -> ClipVisionEncoder:
        return self.encoder

    def encode_image(self, image: ImageInput) -> torch.Tensor:
        return self.encoder.encode(image, getattr(self.engine, "device", None))

    def insert_image_tokens(self, prompt: str, images: int) -> str:
        return insert_image_tokens(prompt, images)

    def fuse_text_and_image_embeddings(self, text: torch.Tensor, image: torch.Tensor) -> torch.Tensor:
        return fuse_text_and_image_embeddings(text, image)

    def image_embeddings(self, image: ImageInput) -> torch.Tensor:
        """[n_patches, hidden]: encoded, then projected into the LM's embedding space."""
        return self.projector(self.encode_image(image))

    def add_request(self, prompt_ids: list[int], image: ImageInput, params=None, image_token_id: int = 0,
                    **kw):
        """Queue ``prompt_ids`` followed by one placeholder token per image patch; the placeholders'
        input embeddings are the projected patches."""
        e = self.image_embeddings(image)
        ids = list(prompt_ids) + [image_token_id] * e.shape[0]
        return self.engine.add_request(ids, params, embeds=(len(prompt_ids), e), **kw)

    def generate(self, prompt_ids: list[int], image: ImageInput, params=None, image_token_id: int = 0):
        s = self.add_request(prompt_ids, image, params, image_token_id)
        while self.engine.has_work():
            self.engine.step()
        return self.engine._result(s)


class LlavaModel(VisionLanguageModel):
    """LLaVA: CLIP ViT-style encoder (224 px, 16 px patches, 768 wide) in front of a llama LM."""

    ARCHES = ("llava", "llama")
    ENCODER = dict(image_size=(224, 224), patch_size=16, embedding_dim=768)


class Qwen2VlModel(VisionLanguageModel):
    """Qwen2-VL: 14 px patches, 1024-wide encoder in front of a qwen2 LM."""

    ARCHES = ("qwen2vl", "qwen2")
    ENCODER = dict(image_size=(224, 224), patch_size=14, embedding_dim=1024)
