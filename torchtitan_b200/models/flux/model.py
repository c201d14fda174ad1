"""FLUX.1 rectified-flow transformer (behaviour parity: reference
``models/flux/model/model.py:25-171`` and ``model/layers.py:24-378``; architecture of
Black Forest Labs' FLUX.1).

Tokens are 2x2 patches of the 16-channel autoencoder latent (64 features each) and
T5 text embeddings.  Conditioning vector ``vec`` = MLP(sinusoidal timestep) +
MLP(CLIP pooled text embedding).

* Double-stream block: image and text tokens keep separate weights (adaptive
  LayerNorm modulation from ``vec``, qkv, per-head RMSNorm of q and k, output
  projection, GELU(tanh) MLP) but attend jointly over ``[text; image]``.
* Single-stream block: one fused ``linear1`` producing qkv and the MLP input of the
  joint sequence, attention, and one ``linear2`` over ``[attention; GELU(mlp)]``.
* Positions: every token has three integer ids (text tokens all zero, image tokens
  (0, row, col)); head dims are split (16, 56, 56) across the three axes and each
  rotates interleaved pairs by ``id * theta^(-2i/d)``: exactly the pairwise
  rotation ``ops.rope`` applies, with per-row tables.

GEMMs run on ``Linear`` (the tcgen05 GEMM on a B200), attention on the flash kernel
(bidirectional), q/k norms on the RMSNorm kernel.
"""
from __future__ import annotations

import dataclasses
import math
from typing import Any

import torch
import torch.nn as nn
import torch.nn.functional as F

from torchtitan_b200 import ops
from torchtitan_b200.protocols import BaseModel, BaseModelArgs
from ..common.layers import Linear, RMSNorm


@dataclasses.dataclass(kw_only=True)
class FluxModelArgs(BaseModelArgs):
    in_channels: int = 64
    out_channels: int = 64
    vec_in_dim: int = 768
    context_in_dim: int = 4096
    hidden_size: int = 3072
    mlp_ratio: float = 4.0
    num_heads: int = 24
    depth: int = 19
    depth_single_blocks: int = 38
    axes_dim: tuple[int, ...] = (16, 56, 56)
    theta: float = 10000.0
    qkv_bias: bool = True
    # autoencoder (the frozen latent encoder/decoder of the images)
    ae_resolution: int = 256
    ae_ch: int = 128
    ae_ch_mult: tuple[int, ...] = (1, 2, 4, 4)
    ae_num_res_blocks: int = 2
    ae_z_channels: int = 16
    ae_scale_factor: float = 0.3611
    ae_shift_factor: float = 0.1159

    def update_from_config(self, trainer_config: Any) -> None:
        pass

    def build(self) -> "FluxModel":
        return FluxModel(self)

    def get_nparams_and_flops(self, model: nn.Module, seq_len: int) -> tuple[int, float]:
        n = sum(p.numel() for p in model.parameters())
        h = self.hidden_size
        # 6 FLOPs per parameter per token plus the two attention matmuls of every block
        return n, 6 * n + 6 * h * seq_len * (self.depth + self.depth_single_blocks)


def timestep_embedding(t: torch.Tensor, dim: int, max_period: float = 10000.0,
                       time_factor: float = 1000.0) -> torch.Tensor:
    """Sinusoidal embedding of ``t * time_factor``: ``[cos(t w_i), sin(t w_i)]`` with
    ``w_i = max_period^(-i / (dim/2))``."""
    t = time_factor * t.float()
    half = dim // 2
    w = torch.exp(-math.log(max_period) * torch.arange(half, dtype=torch.float32, device=t.device) / half)
    a = t[:, None] * w[None]
    emb = torch.cat([torch.cos(a), torch.sin(a)], -1)
    if dim % 2:
        emb = F.pad(emb, (0, 1))
    return emb


def rope_tables(ids: torch.Tensor, axes_dim: tuple[int, ...], theta: float) -> tuple[torch.Tensor, torch.Tensor]:
    """[B, L, n_axes] integer positions -> per-row cos/sin ``[B, L, sum(axes_dim)/2]``."""
    angles = []
    for i, d in enumerate(axes_dim):
        w = theta ** (-torch.arange(0, d, 2, dtype=torch.float64, device=ids.device) / d)
        angles.append(ids[..., i].double()[..., None] * w)
    a = torch.cat(angles, -1)
    return a.cos().float(), a.sin().float()


def _linear(i: int, o: int, init: str, bias: bool = True) -> Linear:
    lin = Linear(i, o, bias=bias)
    lin.flux_init = init
    return lin


class MLPEmbedder(nn.Module):
    def __init__(self, in_dim: int, hidden: int):
        super().__init__()
        self.in_layer = _linear(in_dim, hidden, "normal")
        self.out_layer = _linear(hidden, hidden, "normal")

    def forward(self, x):
        return self.out_layer(F.silu(self.in_layer(x)))


class Modulation(nn.Module):
    """``Linear(SiLU(vec))`` split into (shift, scale, gate) x ``n`` sets, each ``[B, 1, h]``."""

    def __init__(self, h: int, n: int):
        super().__init__()
        self.n = n
        self.lin = _linear(h, 3 * n * h, "zero")

    def forward(self, vec):
        return self.lin(F.silu(vec))[:, None].chunk(3 * self.n, dim=-1)


def _ln(x: torch.Tensor) -> torch.Tensor:
    return F.layer_norm(x, x.shape[-1:], eps=1e-6)


def _attend(q, k, v, cos, sin, cp_group=None):
    """q/k/v [B, L, H, D]: rotary on q and k, bidirectional attention -> [B, L, H*D].
    Under context parallelism (Ulysses) each rank holds a slice of the token sequence:
    an all-to-all trades it for all tokens of H/cp heads around the attention (the order
    of tokens does not matter to bidirectional attention)."""
    q = ops.rope(q.contiguous(), cos, sin)
    k = ops.rope(k.contiguous(), cos, sin)
    v = v.contiguous()
    if cp_group is not None:
        from torchtitan_b200.parallel.context_parallel import head_to_seq, seq_to_head

        q, k, v = (seq_to_head(t, cp_group) for t in (q, k, v))
        return head_to_seq(ops.attention(q, k, v, causal=False), cp_group).flatten(2)
    return ops.attention(q, k, v, causal=False).flatten(2)


class QKNorm(nn.Module):
    def __init__(self, d: int):
        super().__init__()
        self.query_norm = RMSNorm(d, 1e-6)
        self.key_norm = RMSNorm(d, 1e-6)

    def forward(self, q, k, v):
        return self.query_norm(q).to(v.dtype), self.key_norm(k).to(v.dtype)


class StreamAttention(nn.Module):
    def __init__(self, h: int, heads: int, qkv_bias: bool):
        super().__init__()
        self.heads = heads
        self.qkv = _linear(h, 3 * h, "xavier", qkv_bias)
        self.norm = QKNorm(h // heads)
        self.proj = _linear(h, h, "xavier")

    def qkv_heads(self, x):
        B, L, h = x.shape
        q, k, v = self.qkv(x).view(B, L, 3, self.heads, h // self.heads).unbind(2)
        q, k = self.norm(q, k, v)
        return q, k, v


class FluxMLP(nn.Module):
    def __init__(self, h: int, hidden: int):
        super().__init__()
        self.fc1 = _linear(h, hidden, "xavier")
        self.fc2 = _linear(hidden, h, "xavier")

    def forward(self, x):
        return self.fc2(F.gelu(self.fc1(x), approximate="tanh"))


class DoubleStreamBlock(nn.Module):
    cp_group = None  # set by context parallelism

    def __init__(self, h: int, heads: int, mlp_ratio: float, qkv_bias: bool):
        super().__init__()
        mlp = int(h * mlp_ratio)
        self.img_mod, self.txt_mod = Modulation(h, 2), Modulation(h, 2)
        self.img_attn = StreamAttention(h, heads, qkv_bias)
        self.txt_attn = StreamAttention(h, heads, qkv_bias)
        self.img_mlp, self.txt_mlp = FluxMLP(h, mlp), FluxMLP(h, mlp)

    def forward(self, img, txt, vec, cos, sin):
        i_sh1, i_sc1, i_g1, i_sh2, i_sc2, i_g2 = self.img_mod(vec)
        t_sh1, t_sc1, t_g1, t_sh2, t_sc2, t_g2 = self.txt_mod(vec)
        iq, ik, iv = self.img_attn.qkv_heads((1 + i_sc1) * _ln(img) + i_sh1)
        tq, tk, tv = self.txt_attn.qkv_heads((1 + t_sc1) * _ln(txt) + t_sh1)
        o = _attend(torch.cat([tq, iq], 1), torch.cat([tk, ik], 1), torch.cat([tv, iv], 1), cos, sin, self.cp_group)
        t_o, i_o = o[:, :txt.shape[1]], o[:, txt.shape[1]:]
        img = img + i_g1 * self.img_attn.proj(i_o)
        img = img + i_g2 * self.img_mlp((1 + i_sc2) * _ln(img) + i_sh2)
        txt = txt + t_g1 * self.txt_attn.proj(t_o)
        txt = txt + t_g2 * self.txt_mlp((1 + t_sc2) * _ln(txt) + t_sh2)
        return img, txt


class SingleStreamBlock(nn.Module):
    cp_group = None  # set by context parallelism

    def __init__(self, h: int, heads: int, mlp_ratio: float):
        super().__init__()
        self.h, self.heads, self.mlp = h, heads, int(h * mlp_ratio)
        self.linear1 = _linear(h, 3 * h + self.mlp, "xavier")
        self.linear2 = _linear(h + self.mlp, h, "xavier")
        self.norm = QKNorm(h // heads)
        self.modulation = Modulation(h, 1)

    def forward(self, x, vec, cos, sin):
        shift, scale, gate = self.modulation(vec)
        B, L, h = x.shape
        qkv, mlp = self.linear1((1 + scale) * _ln(x) + shift).split([3 * h, self.mlp], -1)
        q, k, v = qkv.reshape(B, L, 3, self.heads, h // self.heads).unbind(2)
        q, k = self.norm(q, k, v)
        o = _attend(q, k, v, cos, sin, self.cp_group)
        return x + gate * self.linear2(torch.cat([o, F.gelu(mlp, approximate="tanh")], -1))


class LastLayer(nn.Module):
    def __init__(self, h: int, out: int):
        super().__init__()
        self.adaLN_modulation = _linear(h, 2 * h, "zero")
        self.linear = _linear(h, out, "zero")

    def forward(self, x, vec):
        shift, scale = self.adaLN_modulation(F.silu(vec))[:, None].chunk(2, -1)
        return self.linear((1 + scale) * _ln(x) + shift)


class FluxModel(BaseModel):
    def __init__(self, a: FluxModelArgs):
        super().__init__()
        self.model_args = a
        h = a.hidden_size
        if h % a.num_heads or sum(a.axes_dim) != h // a.num_heads:
            raise ValueError(f"axes_dim {a.axes_dim} must sum to the head dim {h // a.num_heads}")
        self.img_in = _linear(a.in_channels, h, "xavier")
        self.time_in = MLPEmbedder(256, h)
        self.vector_in = MLPEmbedder(a.vec_in_dim, h)
        self.txt_in = _linear(a.context_in_dim, h, "xavier")
        self.double_blocks = nn.ModuleList(DoubleStreamBlock(h, a.num_heads, a.mlp_ratio, a.qkv_bias)
                                           for _ in range(a.depth))
        self.single_blocks = nn.ModuleList(SingleStreamBlock(h, a.num_heads, a.mlp_ratio)
                                           for _ in range(a.depth_single_blocks))
        self.final_layer = LastLayer(h, a.out_channels)

    def init_weights(self, buffer_device: torch.device | None = None) -> None:
        for m in self.modules():
            if isinstance(m, Linear):
                kind = getattr(m, "flux_init", "xavier")
                if kind == "zero":
                    nn.init.zeros_(m.weight)
                elif kind == "normal":
                    nn.init.normal_(m.weight, std=0.02)
                else:
                    nn.init.xavier_uniform_(m.weight)
                if m.bias is not None:
                    nn.init.zeros_(m.bias)
            elif isinstance(m, RMSNorm):
                m.init_weights()

    def forward(self, img: torch.Tensor, img_ids: torch.Tensor, txt: torch.Tensor, txt_ids: torch.Tensor,
                timesteps: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
        """img [B, L_img, 64] packed latents, txt [B, L_txt, context_in_dim], ids [B, L, 3],
        timesteps [B] in [0, 1], y [B, vec_in_dim] -> predicted velocity [B, L_img, 64]."""
        a = self.model_args
        dt = self.img_in.weight.dtype
        img = self.img_in(img.to(dt))
        vec = self.time_in(timestep_embedding(timesteps, 256).to(dt)) + self.vector_in(y.to(dt))
        txt = self.txt_in(txt.to(dt))
        cos, sin = rope_tables(torch.cat([txt_ids, img_ids], 1), a.axes_dim, a.theta)
        for blk in self.double_blocks:
            img, txt = blk(img, txt, vec, cos, sin)
        x = torch.cat([txt, img], 1)
        for blk in self.single_blocks:
            x = blk(x, vec, cos, sin)
        return self.final_layer(x[:, txt.shape[1]:], vec)
