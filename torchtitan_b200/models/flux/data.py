"""Image-caption batches for FLUX (behaviour parity: reference
``models/flux/flux_datasets.py``): each batch is ``({"captions": [...]}, images)``
with ``images`` ``[B, 3, S, S]`` in [-1, 1]; the trainer encodes both.

``dataset="synthetic"`` draws random images and captions seeded per sample (no
network, reproducible, independent of the batch size); any other value is a local
JSONL file or directory of ``{"image": <path>, "caption": <text>}`` records.
Captions are dropped (replaced by "") with ``prompt_dropout_prob`` so the model
also learns the unconditional velocity used by classifier-free guidance.
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass
from typing import Any, Iterator

import torch
import torch.nn.functional as F

from torchtitan_b200.components.dataloader import BaseDataLoader

_WORDS = ("a photo of", "red", "blue", "small", "large", "cat", "dog", "house", "tree", "on a hill",
          "at night", "in the snow", "painting", "car", "river", "mountain", "city", "portrait")


class FluxDataLoader(BaseDataLoader):
    @dataclass(kw_only=True, slots=True)
    class Config(BaseDataLoader.Config):
        dataset: str = "synthetic"
        img_size: int = 256
        prompt_dropout_prob: float = 0.447
        seed: int = 1234

    def __init__(self, config: Config, **kw: Any):
        super().__init__(config, **kw)
        self.sample_idx = 0

    def _gen(self, sample: int) -> torch.Generator:
        return torch.Generator().manual_seed(hash((self.config.seed, self.dp_rank, sample)) & (2**63 - 1))

    def _synthetic(self, sample: int) -> tuple[torch.Tensor, str]:
        g = self._gen(sample)
        S = self.config.img_size
        low = torch.rand(1, 3, S // 16, S // 16, generator=g) * 2 - 1  # smooth image: upsampled noise
        img = F.interpolate(low, size=(S, S), mode="bilinear", align_corners=False)[0]
        n = int(torch.randint(2, 7, (1,), generator=g))
        cap = " ".join(_WORDS[int(i)] for i in torch.randint(0, len(_WORDS), (n,), generator=g))
        return img, cap

    def _records(self) -> Iterator[tuple[str, str]]:
        p = self.config.dataset
        files = [os.path.join(p, f) for f in sorted(os.listdir(p)) if f.endswith(".jsonl")] if os.path.isdir(p) \
            else [p]
        i = 0
        while True:
            for fn in files:
                with open(fn) as f:
                    for line in f:
                        if line.strip():
                            if i % self.dp_world_size == self.dp_rank:
                                r = json.loads(line)
                                yield os.path.join(os.path.dirname(fn), r["image"]), r.get("caption", "")
                            i += 1

    def _load(self, path: str) -> torch.Tensor:
        from PIL import Image

        S = self.config.img_size
        im = Image.open(path).convert("RGB")
        w, h = im.size
        s = min(w, h)  # center crop to a square, then resize
        im = im.crop(((w - s) // 2, (h - s) // 2, (w - s) // 2 + s, (h - s) // 2 + s)).resize((S, S), Image.BICUBIC)
        x = torch.frombuffer(bytearray(im.tobytes()), dtype=torch.uint8).view(S, S, 3)
        return x.permute(2, 0, 1).float() / 127.5 - 1.0

    def __iter__(self):
        c = self.config
        recs = None
        if c.dataset != "synthetic":
            recs = self._records()
            for _ in range(self.sample_idx * self.local_batch_size):  # resume: skip consumed records
                next(recs)
        while True:
            imgs, caps = [], []
            for j in range(self.local_batch_size):
                sample = self.sample_idx * self.local_batch_size + j
                if recs is None:
                    img, cap = self._synthetic(sample)
                else:
                    path, cap = next(recs)
                    img = self._load(path)
                if float(torch.rand(1, generator=self._gen(-1 - sample))) < c.prompt_dropout_prob:
                    cap = ""
                imgs.append(img)
                caps.append(cap)
            self.sample_idx += 1
            yield {"captions": caps}, torch.stack(imgs)

    def _local_state(self):
        return {"sample_idx": self.sample_idx}

    def _load_local_state(self, st):
        self.sample_idx = int(st["sample_idx"])
