"""Qwen3-VL: the Qwen3 decoder fed with vision tokens (behaviour parity: reference
``models/qwen3_vl/model.py:22-638``; numerics: HF ``Qwen3VLForConditionalGeneration``).

* Every position holding ``image_token_id`` (``video_token_id``) takes, in order, the
  next merged vision token of the encoder.
* DeepStack: the encoder's intermediate features are added at the vision positions
  after each of the first ``len(deepstack_indices)`` decoder layers.
* MRoPE: each token has a (temporal, row, column) position.  Text tokens use their
  running index on all three axes; a vision region of ``t x h x w`` merged tokens
  starting after ``p`` positions gets ``(p + ti, p + hi, p + wi)``, and the text after it
  resumes at ``p + max(t, h, w)``.  Packed documents (``positions`` resetting to 0)
  restart the count.  Rotary frequency ``j`` turns with the row position when
  ``j % 3 == 1`` and ``j < 3 * section[1]``, with the column when ``j % 3 == 2`` and
  ``j < 3 * section[2]``, else with the temporal one.
"""
from __future__ import annotations

import dataclasses
from typing import Any

import torch
import torch.nn as nn

from ..qwen3.model import Qwen3Model, Qwen3ModelArgs
from .vision import Qwen3VLVisionEncoder


@dataclasses.dataclass(kw_only=True)
class Qwen3VLModelArgs(Qwen3ModelArgs):
    rope_theta: float = 5000000.0
    max_seq_len: int = 32768
    mrope_section: tuple[int, int, int] = (24, 20, 20)
    image_token_id: int = 151655
    video_token_id: int = 151656
    vision_dim: int = 1152
    vision_ffn_dim: int = 4304
    vision_layers: int = 27
    vision_heads: int = 16
    patch_size: int = 16
    temporal_patch_size: int = 2
    spatial_merge_size: int = 2
    num_position_embeddings: int = 2304
    deepstack_indices: tuple[int, ...] = (8, 16, 24)

    def build(self) -> "Qwen3VLModel":
        return Qwen3VLModel(self)

    def get_nparams_and_flops(self, model: nn.Module, seq_len: int) -> tuple[int, float]:
        # decoder FLOPs per token (the encoder's depend on the image count of each batch)
        from ..common.blocks import nparams_and_flops

        n, f = nparams_and_flops(model, self.n_layers, self.n_heads, 2 * self.head_dim, seq_len,
                                 self.enable_weight_tying)
        nv = sum(p.numel() for p in model.vision_encoder.parameters())
        return n, f - 6 * nv  # vision parameters do not run per text token


def mrope_positions(tokens: torch.Tensor, image_id: int, video_id: int, image_grids: list, video_grids: list,
                    merge: int, positions: torch.Tensor | None = None) -> torch.Tensor:
    """``[3, B, S]`` (temporal, row, column) positions.  ``image_grids`` / ``video_grids``
    list the (t, h, w) patch grids of the images / videos in token order; a video is
    split into its frames (each its own region, as the reference does).  Consecutive
    placeholder tokens are consumed region by region."""
    B, S = tokens.shape
    ids = tokens.cpu()
    starts_doc = (positions == 0).cpu() if positions is not None else None
    frames = [(1, h, w) for t, h, w in video_grids for _ in range(t)]
    its = {image_id: iter(image_grids), video_id: iter(frames)}
    out = torch.zeros(3, B, S, dtype=torch.long)
    for b in range(B):
        row = ids[b].tolist()
        s, nxt = 0, 0
        while s < S:
            if starts_doc is not None and s > 0 and bool(starts_doc[b, s]):
                nxt = 0
            if row[s] in its:
                t, h, w = next(its[row[s]])
                h, w = h // merge, w // merge
                n = t * h * w
                ti = torch.arange(t).repeat_interleave(h * w)
                hi = torch.arange(h).repeat_interleave(w).repeat(t)
                wi = torch.arange(w).repeat(t * h)
                out[:, b, s:s + n] = (torch.stack([ti, hi, wi]) + nxt)[:, :S - s]
                nxt += max(t, h, w)
                s += n
            else:
                out[:, b, s] = nxt
                nxt += 1
                s += 1
    return out.to(tokens.device)


class Qwen3VLModel(Qwen3Model):
    def __init__(self, a: Qwen3VLModelArgs):
        super().__init__(a)
        self.vision_encoder = Qwen3VLVisionEncoder(
            dim=a.vision_dim, ffn_dim=a.vision_ffn_dim, n_layers=a.vision_layers, n_heads=a.vision_heads,
            patch_size=a.patch_size, temporal_patch_size=a.temporal_patch_size,
            spatial_merge_size=a.spatial_merge_size, out_dim=a.dim,
            num_position_embeddings=a.num_position_embeddings, deepstack_indices=a.deepstack_indices)
        hd2 = a.head_dim // 2
        j = torch.arange(hd2)
        axis = torch.zeros(hd2, dtype=torch.long)
        axis[(j % 3 == 1) & (j < 3 * a.mrope_section[1])] = 1
        axis[(j % 3 == 2) & (j < 3 * a.mrope_section[2])] = 2
        self.register_buffer("mrope_axis", axis, persistent=False)

    def init_weights(self, buffer_device=None) -> None:
        super().init_weights(buffer_device)
        self.vision_encoder.init_weights(buffer_device)
        a = self.model_args
        hd2 = a.head_dim // 2
        j = torch.arange(hd2, device=buffer_device or self.mrope_axis.device)
        axis = torch.zeros_like(j)
        axis[(j % 3 == 1) & (j < 3 * a.mrope_section[1])] = 1
        axis[(j % 3 == 2) & (j < 3 * a.mrope_section[2])] = 2
        self.mrope_axis = axis

    def mrope_tables(self, pos3: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """[3, B, S] positions -> per-row cos/sin ``[B, S, head_dim/2]``."""
        sel = pos3.permute(1, 2, 0)[..., self.mrope_axis]          # [B, S, hd/2]: position driving freq j
        j = torch.arange(sel.shape[-1], device=sel.device)
        return self.rope.cos[sel, j], self.rope.sin[sel, j]

    def forward(self, tokens: torch.Tensor, attention_masks=None, positions: torch.Tensor | None = None,
                pixel_values: torch.Tensor | None = None, grid_thw: torch.Tensor | None = None,
                pixel_values_videos: torch.Tensor | None = None, grid_thw_videos: torch.Tensor | None = None,
                **_: Any) -> torch.Tensor:
        a = self.model_args
        h = self.tok_embeddings(tokens)
        feats, deep = [], None
        img_mask = tokens == a.image_token_id
        vid_mask = tokens == a.video_token_id
        if pixel_values is not None and pixel_values.numel() == 0:
            pixel_values = None
        if pixel_values_videos is not None and pixel_values_videos.numel() == 0:
            pixel_values_videos = None
        for kind, pix, g in (("image", pixel_values, grid_thw), ("video", pixel_values_videos, grid_thw_videos)):
            if pix is None:
                continue
            x, ds = self.vision_encoder(pix, g)
            feats.append((kind, x, ds))
        if not feats and self.training:
            # a batch without images still runs the encoder (on one zero patch block, added
            # with weight 0) so every data-parallel rank issues the same collectives
            m = a.spatial_merge_size
            x, ds = self.vision_encoder(h.new_zeros(m * m, self.vision_encoder.patch_dim),
                                        torch.tensor([[1, m, m]]))
            h = h + 0.0 * (x.sum() + sum(d.sum() for d in ds)).to(h.dtype)
        vis_mask = img_mask | vid_mask
        if feats:
            if len(feats) == 1:
                x, ds = feats[0][1], feats[0][2]
            else:  # interleave image and video tokens in sequence order
                sel = img_mask[vis_mask]
                n, d = int(vis_mask.sum()), feats[0][1].shape[-1]
                x = h.new_zeros(n, d)
                x[sel] = feats[0][1].to(x.dtype)
                x[~sel] = feats[1][1].to(x.dtype)
                ds = []
                for fi, fv in zip(feats[0][2], feats[1][2]):
                    z = h.new_zeros(n, d)
                    z[sel] = fi.to(z.dtype)
                    z[~sel] = fv.to(z.dtype)
                    ds.append(z)
            if x.shape[0] != int(vis_mask.sum()):
                raise ValueError(f"{int(vis_mask.sum())} vision placeholder tokens but {x.shape[0]} vision tokens")
            h = h.masked_scatter(vis_mask[..., None], x.to(h.dtype))
            deep = ds
        if feats:
            pos3 = mrope_positions(tokens, a.image_token_id, a.video_token_id,
                                   grid_thw.tolist() if pixel_values is not None else [],
                                   grid_thw_videos.tolist() if pixel_values_videos is not None else [],
                                   a.spatial_merge_size, positions)
        elif positions is not None:
            pos3 = positions[None].expand(3, *positions.shape)
        else:
            pos3 = torch.arange(tokens.shape[1], device=tokens.device)[None, None].expand(3, tokens.shape[0], -1)
        cos, sin = self.mrope_tables(pos3)
        if deep is not None:
            idx = vis_mask.nonzero(as_tuple=True)
        for i, layer in enumerate(self.layers.values()):
            h = layer(h, cos, sin, attention_masks)
            if deep is not None and i < len(deep):
                h = torch.index_put(h, idx, deep[i].to(h.dtype), accumulate=True)
        h = self.norm(h)
        return self.output(h)
