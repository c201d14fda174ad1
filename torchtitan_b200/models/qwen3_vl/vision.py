"""Qwen3-VL vision encoder (behaviour parity: reference
``models/qwen3_vl/vision_encoder.py:233-704``; numerics: HF ``Qwen3VLVisionModel``).

Input is the processor's flat patch list: ``pixel_values`` ``[N_patches, C*T*P*P]``
(each row one ``T x P x P`` patch of every channel) with ``grid_thw`` ``[N_images, 3]``
giving each image's (frames, patch rows, patch cols).  Patches of an image come in
merge-block order: the ``m x m`` patches that later merge into one LLM token are
consecutive.

* patch embedding: one linear map of the flattened patch (the stride-equals-kernel
  Conv3d of the HF model, as a GEMM);
* learned absolute positions on a ``n x n`` grid, bilinearly resampled to each
  image's ``h x w`` patch grid;
* ViT blocks: LayerNorm, bidirectional attention inside each frame with a 2-D rotary
  embedding (half the rotary frequencies follow the patch row, half the column),
  LayerNorm, GELU(tanh) MLP;
* patch merger: LayerNorm, concatenation of each ``m x m`` block, 2-layer GELU MLP
  to the LLM width; DeepStack mergers (LayerNorm after the concatenation) tap the
  outputs of chosen blocks.

The GEMMs go through ``Linear`` (the tcgen05 GEMM on a B200) and attention through
the flash kernel, one launch per frame (no padding, no cross-image tiles).
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from torchtitan_b200 import ops
from ..common.layers import Linear


class VisionBlock(nn.Module):
    def __init__(self, dim: int, ffn_dim: int, n_heads: int):
        super().__init__()
        self.n_heads = n_heads
        self.norm1 = nn.LayerNorm(dim, eps=1e-6)
        self.norm2 = nn.LayerNorm(dim, eps=1e-6)
        self.qkv = Linear(dim, 3 * dim, bias=True)
        self.proj = Linear(dim, dim, bias=True)
        self.fc1 = Linear(dim, ffn_dim, bias=True)
        self.fc2 = Linear(ffn_dim, dim, bias=True)

    def init_weights(self) -> None:
        for n in (self.norm1, self.norm2):
            n.reset_parameters()
        for lin in (self.qkv, self.proj, self.fc1, self.fc2):
            lin.init_weights(0.02)

    def attention(self, x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, lengths: list[int]) -> torch.Tensor:
        N, D = x.shape
        q, k, v = self.qkv(x).view(N, 3, self.n_heads, D // self.n_heads).unbind(1)
        q = ops.rope(q[None].contiguous(), cos, sin)[0]
        k = ops.rope(k[None].contiguous(), cos, sin)[0]
        outs, s0 = [], 0
        for n in lengths:  # bidirectional attention inside each frame
            outs.append(ops.attention(q[None, s0:s0 + n], k[None, s0:s0 + n], v[None, s0:s0 + n], causal=False)[0])
            s0 += n
        return self.proj(torch.cat(outs).reshape(N, D))

    def forward(self, x, cos, sin, lengths):
        x = x + self.attention(self.norm1(x), cos, sin, lengths)
        return x + self.fc2(F.gelu(self.fc1(self.norm2(x)), approximate="tanh"))


class PatchMerger(nn.Module):
    def __init__(self, dim: int, merge: int, out_dim: int, postshuffle_norm: bool):
        super().__init__()
        self.merged = dim * merge * merge
        self.postshuffle_norm = postshuffle_norm
        self.norm = nn.LayerNorm(self.merged if postshuffle_norm else dim, eps=1e-6)
        self.fc1 = Linear(self.merged, self.merged, bias=True)
        self.fc2 = Linear(self.merged, out_dim, bias=True)

    def init_weights(self) -> None:
        self.norm.reset_parameters()
        self.fc1.init_weights(0.02)
        self.fc2.init_weights(0.02)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x = self.norm(x.reshape(-1, self.merged)) if self.postshuffle_norm else self.norm(x).reshape(-1, self.merged)
        return self.fc2(F.gelu(self.fc1(x)))


class Qwen3VLVisionEncoder(nn.Module):
    def __init__(self, *, dim: int, ffn_dim: int, n_layers: int, n_heads: int, patch_size: int = 16,
                 temporal_patch_size: int = 2, spatial_merge_size: int = 2, out_dim: int = 2048,
                 num_position_embeddings: int = 2304, deepstack_indices: tuple[int, ...] = (), in_channels: int = 3,
                 rope_theta: float = 10000.0):
        super().__init__()
        self.dim, self.n_heads, self.merge = dim, n_heads, spatial_merge_size
        self.patch_dim = in_channels * temporal_patch_size * patch_size * patch_size
        self.patch_embed = Linear(self.patch_dim, dim, bias=True)
        self.pos_embed = nn.Embedding(num_position_embeddings, dim)
        self.grid = int(round(num_position_embeddings ** 0.5))
        self.blocks = nn.ModuleList(VisionBlock(dim, ffn_dim, n_heads) for _ in range(n_layers))
        self.merger = PatchMerger(dim, spatial_merge_size, out_dim, postshuffle_norm=False)
        self.deepstack_indices = tuple(deepstack_indices)
        self.deepstack_mergers = nn.ModuleList(PatchMerger(dim, spatial_merge_size, out_dim, postshuffle_norm=True)
                                               for _ in self.deepstack_indices)
        hd = dim // n_heads
        self.rope_theta = rope_theta
        self.register_buffer("inv_freq", torch.empty(hd // 4), persistent=False)

    def init_buffers(self, buffer_device: torch.device | None = None) -> None:
        q = self.dim // self.n_heads // 2  # rotary dims per axis
        inv = 1.0 / (self.rope_theta ** (torch.arange(0, q, 2, dtype=torch.float32) / q))
        self.inv_freq = inv.to(buffer_device or self.inv_freq.device)

    def init_weights(self, buffer_device: torch.device | None = None) -> None:
        self.init_buffers(buffer_device)
        self.patch_embed.init_weights(0.02)
        nn.init.trunc_normal_(self.pos_embed.weight, std=0.02)
        for b in self.blocks:
            b.init_weights()
        self.merger.init_weights()
        for m in self.deepstack_mergers:
            m.init_weights()

    # ---------------------------------------------------------------- positions
    def _merge_order(self, t: torch.Tensor, T: int, h: int, w: int) -> torch.Tensor:
        """[h*w, ...] row-major grid -> merge-block order, repeated for T frames."""
        m = self.merge
        t = t.view(h // m, m, w // m, m, *t.shape[1:]).transpose(1, 2).reshape(h * w, *t.shape[1:])
        return t.repeat(T, *([1] * (t.dim() - 1)))

    def position_embeddings(self, grid_thw: list[tuple[int, int, int]]) -> torch.Tensor:
        n = self.grid
        W = self.pos_embed.weight
        out = []
        for T, h, w in grid_thw:
            ys = torch.linspace(0, n - 1, h, device=W.device)
            xs = torch.linspace(0, n - 1, w, device=W.device)
            y0, x0 = ys.floor().long(), xs.floor().long()
            y1, x1 = (y0 + 1).clamp(max=n - 1), (x0 + 1).clamp(max=n - 1)
            fy, fx = (ys - y0)[:, None, None], (xs - x0)[None, :, None]
            e = ((1 - fy) * (1 - fx) * W[y0[:, None] * n + x0[None]] + (1 - fy) * fx * W[y0[:, None] * n + x1[None]]
                 + fy * (1 - fx) * W[y1[:, None] * n + x0[None]] + fy * fx * W[y1[:, None] * n + x1[None]])
            out.append(self._merge_order(e.reshape(h * w, -1), T, h, w))
        return torch.cat(out)

    def rope_tables(self, grid_thw: list[tuple[int, int, int]]) -> tuple[torch.Tensor, torch.Tensor]:
        """cos/sin ``[N_patches, head_dim/2]``: the first half of the rotary pairs turn with
        the patch row, the second half with the column."""
        inv = self.inv_freq
        ang = []
        for T, h, w in grid_thw:
            rows = torch.arange(h, device=inv.device, dtype=torch.float32)[:, None].expand(h, w).reshape(-1)
            cols = torch.arange(w, device=inv.device, dtype=torch.float32)[None, :].expand(h, w).reshape(-1)
            a = torch.cat([rows[:, None] * inv, cols[:, None] * inv], -1)
            ang.append(self._merge_order(a, T, h, w))
        a = torch.cat(ang)
        return a.cos(), a.sin()

    def forward(self, pixel_values: torch.Tensor, grid_thw: torch.Tensor) -> tuple[torch.Tensor, list[torch.Tensor]]:
        """-> (merged tokens ``[N_patches / m^2, out_dim]``, DeepStack features, same shape each)."""
        g = [tuple(int(v) for v in r) for r in grid_thw.tolist()]
        x = self.patch_embed(pixel_values.reshape(-1, self.patch_dim).to(self.patch_embed.weight.dtype))
        x = x + self.position_embeddings(g).to(x.dtype)
        cos, sin = self.rope_tables(g)
        lengths = [h * w for T, h, w in g for _ in range(T)]
        deep = []
        for i, blk in enumerate(self.blocks):
            x = blk(x, cos, sin, lengths)
            if i in self.deepstack_indices:
                deep.append(self.deepstack_mergers[self.deepstack_indices.index(i)](x))
        return self.merger(x), deep
