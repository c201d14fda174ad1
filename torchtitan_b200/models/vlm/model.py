"""Llama 3 + SigLIP2 vision-language model with native resolution and aspect ratio
(behaviour parity: reference ``experiments/vlm/model/{model,siglip2}.py``; encoder
numerics: HF ``Siglip2VisionModel``).

Images arrive as a padded batch of patch sequences: ``pixel_values`` ``[N, L, P*P*C]``
(each image's ``h x w`` patches in raster order, then padding) with ``grid_hw``
``[N, 2]``.  The encoder embeds the patches, adds the learned ``n x n`` position
table resampled to each image's ``h x w`` (bilinear, antialiased), and runs
bidirectional pre-LayerNorm ViT blocks over each image's valid patches only (one
flash-attention launch per image: padding costs nothing).  A SiLU MLP projects the
valid patch features to the LLM width; they replace, in order, the ``image_token_id``
positions of the token embeddings.  The rest is the Llama 3 decoder.
"""
from __future__ import annotations

import dataclasses
from typing import Any

import torch
import torch.nn as nn
import torch.nn.functional as F

from torchtitan_b200 import ops
from ..common.layers import Linear
from ..llama3.model import Llama3Model, Llama3ModelArgs


@dataclasses.dataclass(kw_only=True)
class Llama3Siglip2Args(Llama3ModelArgs):
    image_token_id: int = 2047
    vit_dim: int = 1152
    vit_ffn_dim: int = 4304
    vit_layers: int = 27
    vit_heads: int = 16
    patch_size: int = 16
    channels: int = 3
    n_pos_embs: int = 16  # position table is n_pos_embs x n_pos_embs
    vit_eps: float = 1e-6

    def build(self) -> "Llama3Siglip2":
        return Llama3Siglip2(self)

    def get_nparams_and_flops(self, model: nn.Module, seq_len: int) -> tuple[int, float]:
        n, f = super().get_nparams_and_flops(model, seq_len)
        ne = sum(p.numel() for m in (model.encoder, model.projector) for p in m.parameters())
        return n, f - 6 * ne  # encoder FLOPs depend on the images of a batch, not on text tokens


class VitBlock(nn.Module):
    def __init__(self, d: int, ffn: int, heads: int, eps: float):
        super().__init__()
        self.heads = heads
        self.layer_norm1 = nn.LayerNorm(d, eps=eps)
        self.layer_norm2 = nn.LayerNorm(d, eps=eps)
        self.q_proj, self.k_proj, self.v_proj = (Linear(d, d, bias=True) for _ in range(3))
        self.out_proj = Linear(d, d, bias=True)
        self.fc1, self.fc2 = Linear(d, ffn, bias=True), Linear(ffn, d, bias=True)

    def init_weights(self) -> None:
        for n in (self.layer_norm1, self.layer_norm2):
            n.reset_parameters()
        for lin in (self.q_proj, self.k_proj, self.v_proj, self.out_proj, self.fc1, self.fc2):
            nn.init.xavier_uniform_(lin.weight)
            nn.init.zeros_(lin.bias)

    def forward(self, x: torch.Tensor, lengths: list[int]) -> torch.Tensor:
        N, D = x.shape
        h = self.layer_norm1(x)
        q, k, v = (p(h).view(N, self.heads, D // self.heads) for p in (self.q_proj, self.k_proj, self.v_proj))
        outs, s0 = [], 0
        for n in lengths:
            outs.append(ops.attention(q[None, s0:s0 + n], k[None, s0:s0 + n], v[None, s0:s0 + n], causal=False)[0])
            s0 += n
        x = x + self.out_proj(torch.cat(outs).reshape(N, D))
        return x + self.fc2(F.gelu(self.fc1(self.layer_norm2(x)), approximate="tanh"))


class Siglip2Encoder(nn.Module):
    def __init__(self, a: Llama3Siglip2Args):
        super().__init__()
        self.n_pos = a.n_pos_embs
        self.patch_embedding = Linear(a.channels * a.patch_size ** 2, a.vit_dim, bias=True)
        self.position_embedding = nn.Embedding(a.n_pos_embs ** 2, a.vit_dim)
        self.layers = nn.ModuleList(VitBlock(a.vit_dim, a.vit_ffn_dim, a.vit_heads, a.vit_eps)
                                    for _ in range(a.vit_layers))
        self.post_layernorm = nn.LayerNorm(a.vit_dim, eps=a.vit_eps)

    def init_weights(self) -> None:
        nn.init.xavier_uniform_(self.patch_embedding.weight)
        nn.init.zeros_(self.patch_embedding.bias)
        nn.init.normal_(self.position_embedding.weight, std=0.02)
        for blk in self.layers:
            blk.init_weights()
        self.post_layernorm.reset_parameters()

    def positions(self, hw: list[tuple[int, int]]) -> torch.Tensor:
        n = self.n_pos
        table = self.position_embedding.weight.view(n, n, -1).permute(2, 0, 1)[None].float()
        out = []
        for h, w in hw:
            r = F.interpolate(table, size=(h, w), mode="bilinear", align_corners=False, antialias=True)
            out.append(r[0].flatten(1).t())
        return torch.cat(out)

    def forward(self, pixel_values: torch.Tensor, grid_hw: torch.Tensor) -> torch.Tensor:
        """-> valid patch features of every image, concatenated: ``[sum(h*w), vit_dim]``."""
        hw = [tuple(int(v) for v in r) for r in grid_hw.tolist()]
        lengths = [h * w for h, w in hw]
        x = torch.cat([pixel_values[i, :n] for i, n in enumerate(lengths)])
        x = self.patch_embedding(x.to(self.patch_embedding.weight.dtype))
        x = x + self.positions(hw).to(x.dtype)
        for blk in self.layers:
            x = blk(x, lengths)
        return self.post_layernorm(x)


class Projector(nn.Module):
    def __init__(self, din: int, dout: int):
        super().__init__()
        self.w1, self.w2 = Linear(din, din, bias=True), Linear(din, dout, bias=True)

    def init_weights(self) -> None:
        for lin in (self.w1, self.w2):
            nn.init.xavier_uniform_(lin.weight)
            nn.init.zeros_(lin.bias)

    def forward(self, x):
        return self.w2(F.silu(self.w1(x)))


class Llama3Siglip2(Llama3Model):
    def __init__(self, a: Llama3Siglip2Args):
        super().__init__(a)
        self.encoder = Siglip2Encoder(a)
        self.projector = Projector(a.vit_dim, a.dim)

    def init_weights(self, buffer_device=None) -> None:
        super().init_weights(buffer_device)
        self.encoder.init_weights()
        self.projector.init_weights()

    def forward(self, tokens: torch.Tensor, attention_masks=None, positions: torch.Tensor | None = None,
                pixel_values: torch.Tensor | None = None, grid_hw: torch.Tensor | None = None,
                **_: Any) -> torch.Tensor:
        a = self.model_args
        h = self.tok_embeddings(tokens)
        mask = tokens == a.image_token_id
        if pixel_values is not None and pixel_values.numel():
            feats = self.projector(self.encoder(pixel_values, grid_hw))
            if feats.shape[0] != int(mask.sum()):
                raise ValueError(f"{int(mask.sum())} image placeholders but {feats.shape[0]} image patches")
            h = h.masked_scatter(mask[..., None], feats.to(h.dtype))
        elif self.training:  # keep every data-parallel rank's collectives identical
            z = self.projector(self.encoder(h.new_zeros(1, 1, self.encoder.patch_embedding.in_features),
                                            torch.tensor([[1, 1]])))
            h = h + 0.0 * z.sum().to(h.dtype)
        cos, sin = self._rope_tables(tokens.shape[1], positions)
        for layer in self.layers.values():
            h = layer(h, cos, sin, attention_masks)
        return self.output(self.norm(h))
