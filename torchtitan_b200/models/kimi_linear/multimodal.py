"""LLaVA-style multimodal Kimi-Linear (behaviour parity: reference
``experiments/attention_residual/kimi_linear/multimodal_model.py:56-319``).

* a vision tower (pluggable; default a small patch-embedding encoder, any
  module mapping ``[N_img, C, H, W]`` to ``[N_img, patches, vision_dim]`` works,
  e.g. a pretrained SigLIP) -- frozen unless ``train_vision_tower``;
* a 2-layer GELU projector ``vision_dim -> projector_dim -> hidden_size``;
* the Kimi-Linear decoder, fed with token embeddings in which every position
  holding ``vision_token_id`` is replaced, in order, by the next projected
  image patch.

Labels at image positions should be ``IGNORE_INDEX`` (``image_label_mask``
builds them), so only text is trained.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..common.layers import Linear


class PatchVisionTower(nn.Module):
    """Minimal ViT stem: non-overlapping patches -> linear embedding + learned positions."""

    def __init__(self, image_size: int = 224, patch: int = 14, channels: int = 3, dim: int = 1024):
        super().__init__()
        self.patch = patch
        self.proj = nn.Linear(channels * patch * patch, dim)
        self.pos = nn.Parameter(torch.zeros((image_size // patch) ** 2, dim))

    def forward(self, pixels: torch.Tensor) -> torch.Tensor:
        n, c, h, w = pixels.shape
        p = self.patch
        x = pixels.unfold(2, p, p).unfold(3, p, p)                     # [n, c, h/p, w/p, p, p]
        x = x.permute(0, 2, 3, 1, 4, 5).reshape(n, (h // p) * (w // p), c * p * p)
        return self.proj(x) + self.pos[: x.shape[1]]


class VisionProjector(nn.Module):
    def __init__(self, vision_dim: int, projector_dim: int, hidden: int):
        super().__init__()
        self.fc1 = Linear(vision_dim, projector_dim)
        self.fc2 = Linear(projector_dim, hidden)

    def init_weights(self, std: float = 0.02) -> None:
        self.fc1.init_weights(std)
        self.fc2.init_weights(std)

    def forward(self, feats: torch.Tensor) -> torch.Tensor:
        return self.fc2(F.gelu(self.fc1(feats)))


class KimiLinearMultimodal(nn.Module):
    def __init__(self, llm: nn.Module, *, vision_tower: nn.Module | None = None, vision_dim: int = 1024,
                 projector_dim: int = 4096, vision_token_id: int = -200, train_vision_tower: bool = False):
        super().__init__()
        self.llm = llm
        self.vision_tower = vision_tower
        self.vision_token_id = vision_token_id
        hidden = llm.model_args.hidden_size
        self.projector = VisionProjector(vision_dim, projector_dim, hidden)
        if vision_tower is not None and not train_vision_tower:
            for p in vision_tower.parameters():
                p.requires_grad_(False)

    def init_weights(self, buffer_device=None) -> None:
        self.llm.init_weights(buffer_device)
        self.projector.init_weights()

    def embed(self, tokens: torch.Tensor, pixel_values: torch.Tensor | None = None) -> torch.Tensor:
        is_img = tokens == self.vision_token_id
        text = self.llm.embed_tokens(tokens.masked_fill(is_img, 0))
        if pixel_values is None or not bool(is_img.any()):
            if bool(is_img.any()):
                raise ValueError("sequence has image positions but no pixel_values")
            return text
        feats = self.vision_tower(pixel_values.flatten(0, -4))         # [n_img, patches, vision_dim]
        img = self.projector(feats.to(text.dtype)).reshape(-1, text.shape[-1])
        n = int(is_img.sum())
        if img.shape[0] != n:
            raise ValueError(f"{n} image positions but {img.shape[0]} projected patches")
        out = text.clone()
        out[is_img] = img.to(text.dtype)
        return out

    def forward(self, tokens: torch.Tensor, pixel_values: torch.Tensor | None = None, **kw) -> torch.Tensor:
        return self.llm(tokens, inputs_embeds=self.embed(tokens, pixel_values), **kw)


def image_label_mask(labels: torch.Tensor, tokens: torch.Tensor, vision_token_id: int = -200,
                     ignore_index: int = -100) -> torch.Tensor:
    """Labels with image positions (in either the input or the target) ignored."""
    return labels.masked_fill((labels == vision_token_id) | (tokens == vision_token_id), ignore_index)
