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


class MultimodalDataLoader(BaseDataLoader):
    @dataclass(kw_only=True, slots=True)
    class Config(BaseDataLoader.Config):
        image_size: int = 224
        patch_size: int = 14
        vision_token_id: int = -200
        image_marker: str = "<image>"
        pad_id: int = 0
        infinite: bool = True

    def __init__(self, config: Config, **kw: Any):
        super().__init__(config, **kw)
        if config.dataset_path is None:
            raise ValueError("MultimodalDataLoader needs dataset_path (local JSONL)")
        self.ppi = (config.image_size // config.patch_size) ** 2
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
            pix = torch.stack(imgs) if imgs else torch.zeros(0, 3, self.config.image_size, self.config.image_size)
            labels = lab[:, 1:].masked_fill(ids[:, 1:] == self.config.vision_token_id, IGNORE_INDEX)
            yield {"input": ids[:, :-1], "positions": pos[:, :-1], "pixel_values": pix}, labels

    def _local_state(self):
        return {"sample_idx": self.sample_idx}

    def _load_local_state(self, st):
        self.sample_idx = int(st["sample_idx"])
