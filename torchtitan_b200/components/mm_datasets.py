"""Multimodal datasets in the public OBELICS and CC12M formats, with the native-resolution
image pipeline, sample packing and batch collation of Qwen-VL-style training (behaviour
parity: reference ``hf_datasets/multimodal/mm_datasets.py:87-596``,
``mm_collator.py:22-196`` and ``utils/{image,packing,text}.py``).

Sources (local files; there is no network for HF streaming):

* ``obelics`` -- interleaved documents: rows with ``texts`` and ``images`` lists of equal
  length, exactly one of the two set at each position (``None`` in the other).  Read from
  parquet files (pyarrow) or JSONL lines.  An image entry is encoded bytes, a path
  (relative to the file) or, in JSONL, ``{"bytes": <base64>}``.
* ``cc12m`` -- image/caption pairs as WebDataset tar shards: members ``<key>.jpg`` (or
  ``.png``/``.jpeg``/``.webp``) and ``<key>.txt`` grouped by key.
* ``video_frames`` -- JSONL rows ``{"text": ..., "frames": [paths]}`` (a video given as its
  sampled frames; no video decoder is installed), placed before the text.

Each sample becomes ``input_ids`` / ``labels`` (vision placeholder tokens masked with
``IGNORE_INDEX``) / ``positions`` and a list of images ``[T, H, W, C]``: every image is
resized to the pixel budget with both sides multiples of ``patch_size * merge_size``
(``smart_resize``, the published Qwen2-VL resizing rule) and normalised.  An image
contributes ``<vision_start> <image_pad> * n <vision_end>`` with
``n = ceil(T / temporal) * (H / (patch*merge)) * (W / (patch*merge))``.

``SamplePacker`` bin-packs samples into ``seq_len + 1`` sequences by scanning its whole
buffer for samples that still fit; ``MultiModalCollator`` pads text to ``seq_len + 1``,
drops trailing samples beyond ``max_images_per_batch``, shifts inputs/labels and
converts images to the model's flat patch rows (``[sum T'*H'*W', C*temporal*P*P]``, each
``merge x merge`` group consecutive) with ``grid_thw`` rows ``[T', H', W']`` -- the
layout the Qwen3-VL vision tower here consumes.
"""
from __future__ import annotations

import base64
import glob
import io
import json
import math
import os
import tarfile
from collections.abc import Iterator
from dataclasses import dataclass, field
from typing import Any, Callable

import torch

from .dataloader import BaseDataLoader
from .loss import IGNORE_INDEX

# Qwen2/3-VL vocabulary ids of the vision special tokens (used when the tokenizer lacks them)
DEFAULT_SPECIAL = {"vision_start": 151652, "vision_end": 151653, "image": 151655, "video": 151656}
_TOKEN_TEXT = {"vision_start": "<|vision_start|>", "vision_end": "<|vision_end|>", "image": "<|image_pad|>",
               "video": "<|video_pad|>", "pad": "<|endoftext|>"}
_IMAGE_EXT = (".jpg", ".jpeg", ".png", ".webp")


# --------------------------------------------------------------------------- images
def smart_resize(height: int, width: int, factor: int, min_pixels: int, max_pixels: int) -> tuple[int, int]:
    """Target (height, width): both multiples of ``factor``, area within [min_pixels, max_pixels],
    aspect ratio kept as far as the rounding allows (the Qwen2-VL processor's rule)."""
    if max(height, width) > 200 * min(height, width):
        raise ValueError(f"aspect ratio {max(height, width) / min(height, width):.1f} exceeds 200")
    h = max(factor, round(height / factor) * factor)
    w = max(factor, round(width / factor) * factor)
    if h * w > max_pixels:
        s = math.sqrt(height * width / max_pixels)
        h = max(factor, math.floor(height / s / factor) * factor)
        w = max(factor, math.floor(width / s / factor) * factor)
    elif h * w < min_pixels:
        s = math.sqrt(min_pixels / (height * width))
        h = math.ceil(height * s / factor) * factor
        w = math.ceil(width * s / factor) * factor
    return h, w


def decode_image(src: Any, root: str = ""):
    """PIL RGB image from encoded bytes, a path (relative to ``root``), ``{"bytes": ...}`` or PIL."""
    from PIL import Image

    if isinstance(src, dict):
        src = src.get("bytes") if src.get("bytes") is not None else src.get("path")
    if isinstance(src, str) and src.startswith("b64:"):
        src = base64.b64decode(src[4:])
    if isinstance(src, (bytes, bytearray, memoryview)):
        img = Image.open(io.BytesIO(bytes(src)))
    elif isinstance(src, str):
        img = Image.open(src if os.path.isabs(src) else os.path.join(root, src))
    else:
        img = src
    return img.convert("RGB")


@dataclass
class VisionSpec:
    patch_size: int = 16
    temporal_patch_size: int = 2
    merge_size: int = 2
    min_pixels: int = 65536
    max_pixels: int = 16777216
    image_mean: tuple[float, ...] = (0.5, 0.5, 0.5)
    image_std: tuple[float, ...] = (0.5, 0.5, 0.5)

    @property
    def factor(self) -> int:
        return self.patch_size * self.merge_size


def process_frames(frames: list[Any], spec: VisionSpec, root: str = "") -> torch.Tensor:
    """Decode, resize (one size for every frame, from the first) and normalise -> [T, H, W, C] fp32."""
    from PIL import Image

    imgs = [decode_image(f, root) for f in frames]
    w0, h0 = imgs[0].size
    f = spec.factor
    if h0 < f or w0 < f:  # grow tiny images so the rounding has a starting point
        k = max(f / w0, f / h0)
        h0, w0 = int(h0 * k), int(w0 * k)
    h, w = smart_resize(h0, w0, f, spec.min_pixels, spec.max_pixels)
    mean = torch.tensor(spec.image_mean).view(1, 1, 3)
    std = torch.tensor(spec.image_std).view(1, 1, 3)
    out = []
    for im in imgs:
        im = im.resize((w, h), Image.BICUBIC)
        x = torch.frombuffer(bytearray(im.tobytes()), dtype=torch.uint8).view(h, w, 3).float() / 255.0
        out.append((x - mean) / std)
    return torch.stack(out)


def vision_tokens(thwc: torch.Size | tuple[int, ...], spec: VisionSpec) -> int:
    T, H, W = thwc[0], thwc[1], thwc[2]
    return math.ceil(T / spec.temporal_patch_size) * (H // spec.factor) * (W // spec.factor)


def vision_to_patches(x: torch.Tensor, spec: VisionSpec) -> tuple[torch.Tensor, list[int]]:
    """[T, H, W, C] -> (patch rows ``[T'*H'*W', C*temporal*P*P]``, ``[T', H', W']``).

    The time axis is padded to a multiple of the temporal patch by repeating the last frame;
    rows are ordered (t, merge-block row, merge-block column, row in block, column in block)
    and each row flattens (channel, frame, pixel row, pixel column)."""
    T, H, W, C = x.shape
    tp, P, m = spec.temporal_patch_size, spec.patch_size, spec.merge_size
    if T % tp:
        x = torch.cat([x, x[-1:].expand(tp - T % tp, H, W, C)])
        T = x.shape[0]
    gt, gh, gw = T // tp, H // P, W // P
    if gh % m or gw % m:
        raise ValueError(f"patch grid {gh}x{gw} is not a multiple of the merge size {m}")
    x = x.reshape(gt, tp, gh // m, m, P, gw // m, m, P, C)
    x = x.permute(0, 2, 5, 3, 6, 8, 1, 4, 7)  # (t, bh, bw, mh, mw, C, tp, P, P)
    return x.reshape(gt * gh * gw, C * tp * P * P), [gt, gh, gw]


# --------------------------------------------------------------------------- sources
def _files(path: str, exts: tuple[str, ...]) -> list[str]:
    if os.path.isdir(path):
        return sorted(f for e in exts for f in glob.glob(os.path.join(path, f"*{e}")))
    return [path]


def read_obelics(path: str) -> Iterator[dict[str, Any]]:
    for fn in _files(path, (".parquet", ".jsonl")):
        root = os.path.dirname(fn)
        if fn.endswith(".parquet"):
            import pyarrow.parquet as pq

            table = pq.read_table(fn, columns=["texts", "images"])
            for row in table.to_pylist():
                yield {"texts": row["texts"], "images": row["images"], "_root": root}
        else:
            with open(fn) as f:
                for line in f:
                    if line.strip():
                        rec = json.loads(line)
                        imgs = [base64.b64decode(i["bytes"]) if isinstance(i, dict) and "bytes" in i else i
                                for i in rec.get("images", [])]
                        yield {"texts": rec.get("texts", []), "images": imgs, "_root": root}


def read_webdataset(path: str) -> Iterator[dict[str, Any]]:
    """Samples of WebDataset tar shards: members sharing a key (name up to the first dot of
    the base name) form one sample ``{ext: bytes}``."""
    for fn in _files(path, (".tar",)):
        with tarfile.open(fn) as tar:
            key, cur = None, {}
            for mem in tar:
                if not mem.isfile():
                    continue
                base = os.path.basename(mem.name)
                k, _, ext = base.partition(".")
                k = os.path.join(os.path.dirname(mem.name), k)
                if k != key and cur:
                    yield cur
                    cur = {}
                key = k
                cur[ext.lower()] = tar.extractfile(mem).read()
                cur["__key__"] = k
            if cur:
                yield cur


def cc12m_to_interleaved(s: dict[str, Any]) -> dict[str, Any] | None:
    img = next((s[e[1:]] for e in _IMAGE_EXT if e[1:] in s), None)
    if img is None or "txt" not in s:
        return None
    return {"texts": [None, s["txt"].decode("utf-8")], "images": [img, None], "_root": ""}


def read_cc12m(path: str) -> Iterator[dict[str, Any]]:
    for s in read_webdataset(path):
        r = cc12m_to_interleaved(s)
        if r is not None:
            yield r


def read_video_frames(path: str) -> Iterator[dict[str, Any]]:
    for fn in _files(path, (".jsonl",)):
        with open(fn) as f:
            for line in f:
                if line.strip():
                    rec = json.loads(line)
                    yield {"texts": [None, rec.get("text", "")], "videos": [rec["frames"], None],
                           "_root": os.path.dirname(fn)}


MM_SOURCES: dict[str, Callable[[str], Iterator[dict[str, Any]]]] = {
    "obelics": read_obelics,
    "cc12m": read_cc12m,
    "video_frames": read_video_frames,
}


# --------------------------------------------------------------------------- samples
def special_ids(tokenizer: Any, overrides: dict[str, int] | None = None) -> dict[str, int]:
    """Vision special-token ids: the tokenizer's own where its vocabulary has them, else defaults."""
    out = dict(DEFAULT_SPECIAL)
    tok = getattr(tokenizer, "tok", None)
    if tok is not None and hasattr(tok, "token_to_id"):
        for k, t in _TOKEN_TEXT.items():
            if k not in out:
                continue
            i = tok.token_to_id(t)
            if i is not None:
                out[k] = i
    out.update(overrides or {})
    return out


def build_sample(rec: dict[str, Any], tokenizer: Any, spec: VisionSpec, ids: dict[str, int],
                 add_eos: bool = True) -> dict[str, Any] | None:
    """Interleaved record -> tokens with vision placeholders, labels, positions, images.
    Returns None (sample dropped) when the record is malformed or an image cannot be decoded."""
    texts = rec.get("texts") or []
    images = rec.get("images") or [None] * len(texts)
    videos = rec.get("videos") or [None] * len(texts)
    if not texts or not (len(texts) == len(images) == len(videos)):
        return None
    toks: list[int] = []
    mask: list[bool] = []
    pix, vids = [], []
    root = rec.get("_root", "")
    for t, im, vd in zip(texts, images, videos):
        if im is not None or vd is not None:
            try:
                x = process_frames([im] if im is not None else list(vd), spec, root)
            except Exception:  # noqa: BLE001 - undecodable image: drop the sample, as the reference does
                return None
            n = vision_tokens(x.shape, spec)
            pad = ids["image"] if im is not None else ids["video"]
            seg = [ids["vision_start"]] + [pad] * n + [ids["vision_end"]]
            toks += seg
            mask += [True] * len(seg)
            (pix if im is not None else vids).append(x)
        elif t:
            e = tokenizer.encode(t)
            toks += e
            mask += [False] * len(e)
    eos = getattr(tokenizer, "eos_id", None)
    if add_eos and eos is not None:
        toks.append(eos)
        mask.append(False)
    input_ids = torch.tensor(toks, dtype=torch.long)
    labels = input_ids.masked_fill(torch.tensor(mask, dtype=torch.bool), IGNORE_INDEX)
    return {"input_ids": input_ids, "labels": labels, "positions": torch.arange(len(toks)),
            "pixel_values": pix, "pixel_values_videos": vids}


class SamplePacker:
    """Packs samples into sequences of at most ``max_len`` tokens.  Samples wait in a buffer;
    once it holds ``buffer_size`` samples, sequences are formed by scanning the whole buffer
    in arrival order and taking every sample that still fits.  A sequence that is not full
    stays in the buffer for later samples unless ``flush`` or the buffer holds twice
    ``buffer_size`` samples; a sample longer than ``max_len`` alone is dropped."""

    def __init__(self, max_len: int, buffer_size: int = 100):
        self.max_len, self.buffer_size = max_len, buffer_size
        self.buffer: list[dict[str, Any]] = []
        self.ready: list[dict[str, Any]] = []

    def add(self, sample: dict[str, Any]) -> None:
        self.buffer.append(sample)
        if len(self.buffer) >= self.buffer_size:
            self._pack(flush=False)

    def flush(self) -> None:
        self._pack(flush=True)

    def _pack(self, flush: bool) -> None:
        self.buffer = [s for s in self.buffer if len(s["input_ids"]) <= self.max_len]
        while self.buffer:
            take, used = [], 0
            for i, s in enumerate(self.buffer):
                n = len(s["input_ids"])
                if used + n <= self.max_len:
                    take.append(i)
                    used += n
            # a sequence with room left waits for later samples, unless the buffer has grown
            # to twice its size (bounded memory when no combination fills a row exactly)
            if not flush and used < self.max_len and len(self.buffer) < 2 * self.buffer_size:
                return
            chosen = set(take)
            picked = [self.buffer[i] for i in take]
            self.buffer = [s for i, s in enumerate(self.buffer) if i not in chosen]
            self.ready.append(merge_samples(picked))

    def pop(self) -> dict[str, Any] | None:
        return self.ready.pop(0) if self.ready else None

    def state_dict(self) -> dict[str, Any]:
        return {"buffer": list(self.buffer), "ready": list(self.ready)}

    def load_state_dict(self, st: dict[str, Any]) -> None:
        self.buffer, self.ready = list(st["buffer"]), list(st["ready"])


def merge_samples(samples: list[dict[str, Any]]) -> dict[str, Any]:
    return {"input_ids": torch.cat([s["input_ids"] for s in samples]),
            "labels": torch.cat([s["labels"] for s in samples]),
            "positions": torch.cat([s["positions"] for s in samples]),
            "pixel_values": [x for s in samples for x in s["pixel_values"]],
            "pixel_values_videos": [x for s in samples for x in s.get("pixel_values_videos", [])]}


@dataclass
class MultiModalCollator:
    batch_size: int
    seq_len: int
    spec: VisionSpec = field(default_factory=VisionSpec)
    max_images_per_batch: int = 1 << 30
    pad_id: int = 0
    special: dict[str, int] = field(default_factory=lambda: dict(DEFAULT_SPECIAL))

    @staticmethod
    def _n_vision(s: dict[str, Any], tp: int) -> int:
        return len(s["pixel_values"]) + sum(math.ceil(v.shape[0] / tp) for v in s.get("pixel_values_videos", []))

    def _patches(self, xs: list[torch.Tensor]) -> tuple[torch.Tensor | None, torch.Tensor | None]:
        if not xs:
            return None, None
        pg = [vision_to_patches(x, self.spec) for x in xs]
        return torch.cat([p for p, _ in pg]), torch.tensor([g for _, g in pg], dtype=torch.long)

    def __call__(self, batch: list[dict[str, Any]]) -> tuple[dict[str, Any], torch.Tensor]:
        batch = list(batch)
        tp = self.spec.temporal_patch_size
        while batch and sum(self._n_vision(s, tp) for s in batch) > self.max_images_per_batch:
            batch.pop()  # the trailing samples go first, as many as needed
        L = self.seq_len + 1
        B = self.batch_size
        ids = torch.full((B, L), self.pad_id, dtype=torch.long)
        lab = torch.full((B, L), IGNORE_INDEX, dtype=torch.long)
        pos = torch.zeros((B, L), dtype=torch.long)
        for i, s in enumerate(batch):
            n = min(L, len(s["input_ids"]))
            ids[i, :n] = s["input_ids"][:n]
            lab[i, :n] = s["labels"][:n]
            pos[i, :n] = s["positions"][:n]
        pix, grid = self._patches([x for s in batch for x in s["pixel_values"]])
        vpix, vgrid = self._patches([x for s in batch for x in s.get("pixel_values_videos", [])])
        out = {"input": ids[:, :-1], "positions": pos[:, :-1], "pixel_values": pix, "grid_thw": grid,
               "pixel_values_videos": vpix, "grid_thw_videos": vgrid,
               "special_tokens": {f"{k}_id": v for k, v in self.special.items()}}
        return out, lab[:, 1:]


# --------------------------------------------------------------------------- loader
class MMDataLoader(BaseDataLoader):
    """Stateful, data-parallel-aware multimodal loader over ``MM_SOURCES`` (records are dealt
    round-robin to the dp ranks); resumes from its record counter and packer state."""

    @dataclass(kw_only=True, slots=True)
    class Config(BaseDataLoader.Config):
        dataset: str = "cc12m"
        infinite: bool = True
        packing_buffer_size: int = 0
        """> 0 packs samples (``SamplePacker``) with this many buffered samples."""
        max_images_per_batch: int = 64
        patch_size: int = 16
        temporal_patch_size: int = 2
        spatial_merge_size: int = 2
        min_pixels: int = 65536
        max_pixels: int = 16777216
        image_mean: tuple[float, ...] = (0.5, 0.5, 0.5)
        image_std: tuple[float, ...] = (0.5, 0.5, 0.5)
        image_token_id: int = -1
        """Placeholder ids (-1: the tokenizer's own token, else the Qwen-VL vocabulary's id)."""
        video_token_id: int = -1
        vision_start_id: int = -1
        vision_end_id: int = -1

    def __init__(self, config: Config, **kw: Any):
        super().__init__(config, **kw)
        if config.dataset not in MM_SOURCES:
            raise ValueError(f"unknown multimodal dataset {config.dataset!r}; known: {sorted(MM_SOURCES)}")
        if config.dataset_path is None:
            raise ValueError("MMDataLoader needs dataset_path (local files)")
        c = config
        self.spec = VisionSpec(c.patch_size, c.temporal_patch_size, c.spatial_merge_size, c.min_pixels,
                               c.max_pixels, tuple(c.image_mean), tuple(c.image_std))
        self.special = special_ids(self.tokenizer, {k: v for k, v in (
            ("image", c.image_token_id), ("video", c.video_token_id), ("vision_start", c.vision_start_id),
            ("vision_end", c.vision_end_id)) if v >= 0})
        pad = getattr(self.tokenizer, "pad_id", None)
        if pad is None:  # the tokenizer's end-of-text token where its vocabulary has one, else id 0
            tok = getattr(self.tokenizer, "tok", None)
            pad = tok.token_to_id(_TOKEN_TEXT["pad"]) if tok is not None and hasattr(tok, "token_to_id") else None
        self.collate = MultiModalCollator(self.local_batch_size, self.seq_len, self.spec, c.max_images_per_batch,
                                          pad if pad is not None else 0, self.special)
        self.packer = SamplePacker(self.seq_len + 1, c.packing_buffer_size) if c.packing_buffer_size > 0 else None
        self.records_seen = 0  # records of the whole stream (all ranks) consumed by this rank's iterator
        self.epoch = 0

    def _samples(self) -> Iterator[dict[str, Any]]:
        read = MM_SOURCES[self.config.dataset]
        while True:
            for i, rec in enumerate(read(self.config.dataset_path)):
                if i < self.records_seen:
                    continue
                self.records_seen = i + 1
                if i % self.dp_world_size != self.dp_rank:
                    continue
                s = build_sample(rec, self.tokenizer, self.spec, self.special)
                if s is None or len(s["input_ids"]) > self.seq_len + 1:
                    continue
                yield s
            self.records_seen = 0
            self.epoch += 1
            if not self.config.infinite:
                return

    def __iter__(self):
        batch: list[dict[str, Any]] = []
        src = self._samples()
        while True:
            if self.packer is not None:
                s = self.packer.pop()
                if s is None:
                    nxt = next(src, None)
                    if nxt is None:
                        self.packer.flush()
                        s = self.packer.pop()
                        if s is None:
                            break
                    else:
                        self.packer.add(nxt)
                        continue
            else:
                s = next(src, None)
                if s is None:
                    break
            batch.append(s)
            if len(batch) == self.local_batch_size:
                yield self.collate(batch)
                batch = []
        if batch:
            yield self.collate(batch)

    def _local_state(self) -> dict[str, Any]:
        st = {"records_seen": self.records_seen, "epoch": self.epoch}
        if self.packer is not None:
            st["packer"] = self.packer.state_dict()
        return st

    def _load_local_state(self, st: dict[str, Any]) -> None:
        self.records_seen, self.epoch = int(st["records_seen"]), int(st["epoch"])
        if self.packer is not None and "packer" in st:
            self.packer.load_state_dict(st["packer"])
