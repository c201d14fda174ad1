"""Interleaved image-text data (behaviour parity: reference
``hf_datasets/multimodal/mm_datasets.py:87,301,482`` and ``mm_collator.py``).

Records are JSONL lines ``{"text": "... <image> ...", "images": ["a.png", ...]}``
(paths relative to the file).  Each ``<image>`` marker becomes
``patches_per_image`` copies of ``vision_token_id`` and consumes the next image,
which is resized to ``image_size`` x ``image_size`` and normalised.  Samples
are packed greedily into ``seq_len + 1`` windows without splitting a sample
(an over-long sample is dropped); labels at image positions and padding are
``IGNORE_INDEX``.  Each batch yields ``{"input", "positions", "pixel_values"}``
where ``pixel_values`` is ``[n_images, 3, H, W]`` in order of appearance, the
order the multimodal model consumes them.

With ``vision_layout="patches"`` (Qwen3-VL style native patches) each image
becomes ``(image_size / patch_size / merge_size)^2`` placeholder tokens and the
batch carries ``pixel_values`` as flat patches ``[n_images * gh * gw, 3*T*P*P]``
(``patchify``) plus ``grid_thw`` ``[n_images, 3]``.
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass
from typing import Any, Iterator

import torch

from .dataloader import BaseDataLoader
from .loss import IGNORE_INDEX

_MEAN = torch.tensor([0.5, 0.5, 0.5]).view(3, 1, 1)
_STD = torch.tensor([0.5, 0.5, 0.5]).view(3, 1, 1)


def load_image(path: str, size: int) -> torch.Tensor:
    from PIL import Image

    img = Image.open(path).convert("RGB").resize((size, size), Image.BICUBIC)
    x = torch.frombuffer(bytearray(img.tobytes()), dtype=torch.uint8).view(size, size, 3)
    return ((x.permute(2, 0, 1).float() / 255.0) - _MEAN) / _STD


def patchify(img: torch.Tensor, patch: int, temporal: int = 2, merge: int = 2) -> tuple[torch.Tensor, list[int]]:
    """[C, H, W] image -> (flat patches ``[gh*gw, C*T*P*P]`` in merge-block order, [1, gh, gw]).

    The image is repeated over the ``temporal`` patch depth; each row holds one
    patch as (channel, frame, row, column); the ``merge x merge`` patches that merge
    into one LLM token are consecutive (the HF Qwen3-VL processor's layout)."""
    C, H, W = img.shape
    gh, gw = H // patch, W // patch
    if gh % merge or gw % merge:
        raise ValueError(f"patch grid {gh}x{gw} is not a multiple of the merge size {merge}")
    x = img[:, : gh * patch, : gw * patch][:, None].expand(C, temporal, gh * patch, gw * patch)
    x = x.reshape(C, temporal, gh // merge, merge, patch, gw // merge, merge, patch)
    x = x.permute(2, 5, 3, 6, 0, 1, 4, 7)  # (bh, bw, mh, mw, C, T, P, P)
    return x.reshape(gh * gw, C * temporal * patch * patch), [1, gh, gw]


def patchify_raster(img: torch.Tensor, patch: int) -> tuple[torch.Tensor, list[int]]:
    """[C, H, W] -> (patches in raster order ``[gh*gw, P*P*C]``, each flattened as (row,
    column, channel): the SigLIP2 processor layout), [gh, gw]."""
    C, H, W = img.shape
    gh, gw = H // patch, W // patch
    x = img[:, : gh * patch, : gw * patch].reshape(C, gh, patch, gw, patch).permute(1, 3, 2, 4, 0)
    return x.reshape(gh * gw, patch * patch * C), [gh, gw]


class MultimodalDataLoader(BaseDataLoader):
    @dataclass(kw_only=True, slots=True)
    class Config(BaseDataLoader.Config):
        image_size: int = 224
        patch_size: int = 14
        vision_token_id: int = -200
        image_marker: str = "<image>"
        pad_id: int = 0
        infinite: bool = True
        vision_layout: str = "images"  # or "patches" (flat native patches + grid_thw)
        temporal_patch_size: int = 2
        merge_size: int = 2

    def __init__(self, config: Config, **kw: Any):
        super().__init__(config, **kw)
        if config.dataset_path is None:
            raise ValueError("MultimodalDataLoader needs dataset_path (local JSONL)")
        g = config.image_size // config.patch_size
        self.ppi = g * g if config.vision_layout == "images" else (g // config.merge_size) ** 2
        self.sample_idx = 0

    def _records(self) -> Iterator[tuple[dict, str]]:
        p = self.config.dataset_path
        files = [os.path.join(p, f) for f in sorted(os.listdir(p)) if f.endswith(".jsonl")] if os.path.isdir(p) \
            else [p]
        while True:
            i = 0
            for fn in files:
                with open(fn) as f:
                    for line in f:
                        if not line.strip():
                            continue
                        if i % self.dp_world_size == self.dp_rank:
                            yield json.loads(line), os.path.dirname(fn)
                        i += 1
            if not self.config.infinite:
                return

    def _sample(self, rec: dict, root: str) -> tuple[list[int], list[int], list[torch.Tensor]]:
        c = self.config
        parts = rec["text"].split(c.image_marker)
        images = rec.get("images", [])
        if len(images) != len(parts) - 1:
            raise ValueError(f"{len(parts) - 1} image markers but {len(images)} images")
        ids, labels, pix = [], [], []
        bos = getattr(self.tokenizer, "bos_id", None)
        if bos is not None:
            ids.append(bos)
            labels.append(bos)
        for k, text in enumerate(parts):
            t = self.tokenizer.encode(text) if text else []
            ids += t
            labels += t
            if k < len(images):
                ids += [c.vision_token_id] * self.ppi
                labels += [IGNORE_INDEX] * self.ppi
                pix.append(load_image(os.path.join(root, images[k]), c.image_size))
        eos = getattr(self.tokenizer, "eos_id", None)
        if eos is not None:
            ids.append(eos)
            labels.append(eos)
        return ids, labels, pix

    def _windows(self):
        W = self.seq_len + 1
        ids, lab, pos, pix = [], [], [], []
        for rec, root in self._records():
            s_ids, s_lab, s_pix = self._sample(rec, root)
            if len(s_ids) > W:
                continue
            if len(ids) + len(s_ids) > W:
                pad = W - len(ids)
                yield ids + [self.config.pad_id] * pad, lab + [IGNORE_INDEX] * pad, pos + list(range(pad)), pix
                ids, lab, pos, pix = [], [], [], []
            ids, lab, pix = ids + s_ids, lab + s_lab, pix + s_pix
            pos += list(range(len(s_ids)))
        if ids:
            pad = W - len(ids)
            yield ids + [self.config.pad_id] * pad, lab + [IGNORE_INDEX] * pad, pos + list(range(pad)), pix

    def __iter__(self):
        batch, skipped = [], 0
        for w in self._windows():
            batch.append(w)
            if len(batch) < self.local_batch_size:
                continue
            ids = torch.tensor([b[0] for b in batch])
            lab = torch.tensor([b[1] for b in batch])
            pos = torch.tensor([b[2] for b in batch])
            imgs = [im for b in batch for im in b[3]]
            batch = []
            if skipped < self.sample_idx:
                skipped += 1
                continue
            self.sample_idx += 1
            skipped += 1
            c = self.config
            labels = lab[:, 1:].masked_fill(ids[:, 1:] == c.vision_token_id, IGNORE_INDEX)
            out = {"input": ids[:, :-1], "positions": pos[:, :-1]}
            if c.vision_layout == "patches":
                pg = [patchify(im, c.patch_size, c.temporal_patch_size, c.merge_size) for im in imgs]
                dim = 3 * c.temporal_patch_size * c.patch_size ** 2
                out["pixel_values"] = torch.cat([p for p, _ in pg]) if pg else torch.zeros(0, dim)
                out["grid_thw"] = torch.tensor([g for _, g in pg], dtype=torch.long).view(-1, 3)
            else:
                out["pixel_values"] = torch.stack(imgs) if imgs else torch.zeros(0, 3, c.image_size, c.image_size)
            yield out, labels

    def _local_state(self):
        return {"sample_idx": self.sample_idx}

    def _load_local_state(self, st):
        self.sample_idx = int(st["sample_idx"])


class SyntheticImageTextDataLoader(BaseDataLoader):
    """Random tokens with ``images_per_sample`` random images per sample, in the
    native-patch layout (``pixel_values`` flat patches + ``grid_thw``); each image's
    placeholder run starts at a random position.  Seeded per sample like
    ``SyntheticDataLoader``."""

    @dataclass(kw_only=True, slots=True)
    class Config(BaseDataLoader.Config):
        vocab_size: int = 0
        seed: int = 1234
        images_per_sample: int = 1
        image_size: int = 256
        patch_size: int = 16
        temporal_patch_size: int = 2
        merge_size: int = 2
        vision_token_id: int = 151655
        layout: str = "patches"
        """"patches": flat merge-ordered patches + ``grid_thw`` (Qwen3-VL);
        "padded": ``[N, L, P*P*C]`` raster patches padded to L = (image_size/P)^2 + ``grid_hw`` (SigLIP2)."""

    def __init__(self, config: Config, **kw: Any):
        super().__init__(config, **kw)
        v = config.vocab_size or kw.get("vocab_size") or (self.tokenizer.get_vocab_size() if self.tokenizer else 2048)
        self.vocab_size = int(v)
        g = config.image_size // config.patch_size
        self.grid = [1, g, g]
        self.tokens_per_image = g * g if config.layout == "padded" else (g // config.merge_size) ** 2
        self.batches_emitted = 0
        if config.images_per_sample * self.tokens_per_image > self.seq_len:
            raise ValueError("images do not fit the sequence")

    def _batch(self, index: int):
        c = self.config
        ids, pix = [], []
        n_text = self.vocab_size - 2 if c.vision_token_id >= self.vocab_size - 2 else self.vocab_size
        for j in range(self.local_batch_size):
            sample = index * self.local_batch_size + j
            g = torch.Generator().manual_seed(hash((c.seed, self.dp_rank, sample)) & (2**63 - 1))
            row = torch.randint(0, n_text, (self.seq_len + 1,), generator=g)
            row[row == c.vision_token_id] = 0
            free = self.seq_len - c.images_per_sample * self.tokens_per_image
            cuts = torch.sort(torch.randint(0, free + 1, (c.images_per_sample,), generator=g)).values.tolist()
            for k, cut in enumerate(cuts):  # k images already placed before this one
                s = cut + k * self.tokens_per_image
                row[s:s + self.tokens_per_image] = c.vision_token_id
                img = torch.randn(3, c.image_size, c.image_size, generator=g)
                if c.layout == "padded":
                    pix.append(patchify_raster(img, c.patch_size)[0])
                else:
                    pix.append(patchify(img, c.patch_size, c.temporal_patch_size, c.merge_size)[0])
            ids.append(row)
        ids = torch.stack(ids)
        labels = ids[:, 1:].masked_fill(ids[:, 1:] == c.vision_token_id, IGNORE_INDEX)
        n = c.images_per_sample * self.local_batch_size
        if c.layout == "padded":
            return ({"input": ids[:, :-1], "pixel_values": torch.stack(pix),
                     "grid_hw": torch.tensor([self.grid[1:]] * n, dtype=torch.long)}, labels)
        return ({"input": ids[:, :-1], "pixel_values": torch.cat(pix),
                 "grid_thw": torch.tensor([self.grid] * n, dtype=torch.long)}, labels)

    def __iter__(self):
        while True:
            b = self._batch(self.batches_emitted)
            self.batches_emitted += 1
            yield b

    def _local_state(self):
        return {"batches_emitted": self.batches_emitted}

    def _load_local_state(self, st):
        self.batches_emitted = int(st["batches_emitted"])
