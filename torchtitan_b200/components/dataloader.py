"""Data loading.

* ``BaseDataLoader`` -- Stateful, DP-aware iterator protocol yielding
  ``({"input": int64[B,S], ...}, labels int64[B,S])`` on the host; state is
  stored per dp rank (parity: ``torchtitan/components/dataloader.py:32-167``).
* ``SyntheticDataLoader`` -- iid uniform tokens in ``[0, vocab)`` from a seed,
  distinct per dp rank and step, resumable from its sample counter.  Batches
  are produced in pinned host memory so the host-to-device copy is async.
* ``HuggingFaceTextDataLoader`` -- tokenises local text/JSONL files (or a
  ``datasets`` dataset saved to disk), greedily concatenates documents into
  ``seq_len + 1`` windows and emits per-document ``positions`` (parity:
  ``torchtitan/hf_datasets/text_datasets.py:72-207``).
"""
from __future__ import annotations

import glob
import json
import os
import pickle
from abc import ABC, abstractmethod
from collections.abc import Iterator
from dataclasses import dataclass
from typing import Any

import torch
from torch.distributed.checkpoint.stateful import Stateful

from torchtitan_b200.config import Configurable


class DataloaderExhaustedError(Exception):
    """Raised by the trainer's batch generator when the data runs out."""


def _local_tensor_mode_active() -> bool:
    try:
        from torch.distributed._local_tensor import local_tensor_mode
    except ImportError:
        return False
    return local_tensor_mode() is not None


def _simulated_ranks(dp_rank: Any) -> dict[int, int] | None:
    """``{global rank: dp rank}`` when ``dp_rank`` is a per-rank integer of LocalTensorMode, else None."""
    if isinstance(dp_rank, torch.SymInt):
        local = getattr(dp_rank.node, "_local_ints", None)
        if local is not None:
            return dict(local)
    return None


class BaseDataLoader(Stateful, ABC, Configurable):
    @dataclass(kw_only=True, slots=True)
    class Config(Configurable.Config):
        dataset: str = "synthetic"
        dataset_path: str | None = None

    def __init__(self, config: Config, *, dp_world_size: int = 1, dp_rank: int = 0, tokenizer: Any = None,
                 seq_len: int = 2048, local_batch_size: int = 1, **kw: Any):
        self.config = config
        self.dp_world_size, self.dp_rank = dp_world_size, dp_rank
        self.tokenizer = tokenizer
        self.seq_len, self.local_batch_size = seq_len, local_batch_size
        self._rank_key = f"dp_rank_{dp_rank}"

    @abstractmethod
    def __iter__(self) -> Iterator[tuple[dict[str, torch.Tensor], torch.Tensor]]:
        ...

    @abstractmethod
    def _local_state(self) -> dict[str, Any]:
        ...

    @abstractmethod
    def _load_local_state(self, st: dict[str, Any]) -> None:
        ...

    def state_dict(self) -> dict[str, Any]:
        return {self._rank_key: pickle.dumps(self._local_state()), "world_size": self.dp_world_size}

    def load_state_dict(self, sd: dict[str, Any]) -> None:
        if not sd:
            return
        if sd.get("world_size", self.dp_world_size) != self.dp_world_size:
            raise ValueError("dataloader state was saved with a different dp degree; resharding is unsupported")
        if self._rank_key in sd:
            self._load_local_state(pickle.loads(sd[self._rank_key]))


class SyntheticDataLoader(BaseDataLoader):
    @dataclass(kw_only=True, slots=True)
    class Config(BaseDataLoader.Config):
        dataset: str = "synthetic"
        vocab_size: int = 0
        """0 = take the vocab size from the tokenizer / model."""
        seed: int = 1234
        max_samples: int = -1
        """Stop after this many batches per rank (-1 = infinite)."""
        pin_memory: bool = True

    def __init__(self, config: Config, **kw: Any):
        super().__init__(config, **kw)
        v = config.vocab_size
        if v <= 0:
            v = kw.get("vocab_size") or (self.tokenizer.get_vocab_size() if self.tokenizer is not None else 2048)
        self.vocab_size = int(v)
        self.batches_emitted = 0

    def _batch(self, index: int) -> torch.Tensor:
        if not _local_tensor_mode_active():
            return self._batch_for(index, self.dp_rank)
        # one process simulating every rank (comm mode local_tensor): the host batch is drawn
        # outside the mode (inside it every rank would draw its own random numbers); with
        # several dp ranks each rank's batch becomes one shard of a LocalTensor
        from torch.distributed._local_tensor import LocalTensor, maybe_disable_local_tensor_mode

        ranks = _simulated_ranks(self.dp_rank)
        with maybe_disable_local_tensor_mode():
            if ranks is None:
                return self._batch_for(index, int(self.dp_rank))
            return LocalTensor({r: self._batch_for(index, d) for r, d in ranks.items()})

    def _batch_for(self, index: int, dp_rank: int) -> torch.Tensor:
        # every sample is seeded by its own index, so the token stream does not depend on how it
        # is cut into batches (a batch of 4 equals two consecutive batches of 2)
        rows = []
        for j in range(self.local_batch_size):
            sample = index * self.local_batch_size + j
            g = torch.Generator().manual_seed(hash((self.config.seed, dp_rank, sample)) & (2**63 - 1))
            rows.append(torch.randint(0, self.vocab_size, (self.seq_len + 1,), generator=g))
        t = torch.stack(rows)
        if self.config.pin_memory and torch.cuda.is_available():
            t = t.pin_memory()
        return t

    def __iter__(self):
        while self.config.max_samples < 0 or self.batches_emitted < self.config.max_samples:
            t = self._batch(self.batches_emitted)
            self.batches_emitted += 1
            yield {"input": t[:, :-1]}, t[:, 1:]

    def _local_state(self):
        return {"batches_emitted": self.batches_emitted}

    def _load_local_state(self, st):
        self.batches_emitted = int(st["batches_emitted"])


def _iter_local_texts(path: str) -> Iterator[str]:
    files = sorted(glob.glob(os.path.join(path, "**", "*"), recursive=True)) if os.path.isdir(path) else [path]
    for fn in files:
        if fn.endswith((".jsonl", ".json")):
            with open(fn) as f:
                for line in f:
                    line = line.strip()
                    if line:
                        yield json.loads(line).get("text", "")
        elif fn.endswith(".txt"):
            with open(fn) as f:
                yield f.read()
        elif os.path.isdir(fn) and os.path.exists(os.path.join(fn, "dataset_info.json")):
            import datasets

            for row in datasets.load_from_disk(fn):
                yield row["text"]


class HuggingFaceTextDataLoader(BaseDataLoader):
    @dataclass(kw_only=True, slots=True)
    class Config(BaseDataLoader.Config):
        dataset: str = "c4_test"
        infinite: bool = True

    def __init__(self, config: Config, **kw: Any):
        super().__init__(config, **kw)
        if config.dataset_path is None:
            raise ValueError("HuggingFaceTextDataLoader needs dataset_path (no network access to fetch datasets)")
        self.sample_idx = 0
        self.buffer: list[int] = []
        self.pos_buffer: list[int] = []

    def _docs(self) -> Iterator[list[int]]:
        while True:
            for i, text in enumerate(_iter_local_texts(self.config.dataset_path)):
                if i % self.dp_world_size != self.dp_rank:
                    continue
                yield self.tokenizer.encode(text, add_bos=True, add_eos=True)
            if not self.config.infinite:
                return

    def __iter__(self):
        need = self.local_batch_size * (self.seq_len + 1)
        skipped = 0
        for doc in self._docs():
            self.buffer.extend(doc)
            self.pos_buffer.extend(range(len(doc)))
            while len(self.buffer) >= need:
                toks = torch.tensor(self.buffer[:need]).view(self.local_batch_size, -1)
                pos = torch.tensor(self.pos_buffer[:need]).view(self.local_batch_size, -1)
                self.buffer, self.pos_buffer = self.buffer[need:], self.pos_buffer[need:]
                if skipped < self.sample_idx:  # fast-forward after a resume
                    skipped += 1
                    continue
                self.sample_idx += 1
                skipped += 1
                yield {"input": toks[:, :-1], "positions": pos[:, :-1]}, toks[:, 1:]

    def _local_state(self):
        return {"sample_idx": self.sample_idx}

    def _load_local_state(self, st):
        self.sample_idx = int(st["sample_idx"])


def _iter_local_records(path: str) -> Iterator[dict]:
    files = sorted(glob.glob(os.path.join(path, "**", "*.jsonl"), recursive=True)) if os.path.isdir(path) else [path]
    for fn in files:
        with open(fn) as f:
            for line in f:
                line = line.strip()
                if line:
                    yield json.loads(line)


def render_chat(messages: list[dict], template: str | None = None) -> list[tuple[str, bool]]:
    """Split a conversation into (text, trainable) segments.  With a jinja
    ``template`` (the tokenizer's chat template) each message is rendered
    alone; otherwise a plain ``<|role|>\\ncontent\\n`` layout is used.  Only
    assistant turns are trainable."""
    out = []
    for m in messages:
        if template:
            import jinja2

            text = jinja2.Template(template).render(messages=[m], add_generation_prompt=False)
        else:
            text = f"<|{m['role']}|>\n{m['content']}\n"
        out.append((text, m["role"] == "assistant"))
    return out


class ChatDataLoader(BaseDataLoader):
    """Supervised fine-tuning data (parity: reference ``hf_datasets/text_datasets.py:262-408``
    ``ChatDataset``): JSONL records with ``messages: [{role, content}, ...]`` are
    tokenised turn by turn, labels of non-assistant tokens are ``IGNORE_INDEX``,
    and samples are greedily packed into ``seq_len + 1`` windows (a sample that
    does not fit starts a new window, padded with ``pad_id`` / ignored labels;
    one longer than the window is truncated).  ``positions`` restart at every
    sample so document-masked attention sees sample boundaries."""

    @dataclass(kw_only=True, slots=True)
    class Config(BaseDataLoader.Config):
        infinite: bool = True
        pad_id: int = 0
        chat_template: str | None = None

    def __init__(self, config: Config, **kw: Any):
        super().__init__(config, **kw)
        if config.dataset_path is None:
            raise ValueError("ChatDataLoader needs dataset_path (local JSONL with a 'messages' field)")
        self.sample_idx = 0

    def _samples(self) -> Iterator[tuple[list[int], list[int]]]:
        from .loss import IGNORE_INDEX

        while True:
            for i, rec in enumerate(_iter_local_records(self.config.dataset_path)):
                if i % self.dp_world_size != self.dp_rank:
                    continue
                ids, labels = [], []
                bos = getattr(self.tokenizer, "bos_id", None)
                if bos is not None:
                    ids.append(bos)
                    labels.append(IGNORE_INDEX)
                for text, train in render_chat(rec["messages"], self.config.chat_template):
                    t = self.tokenizer.encode(text)
                    ids += t
                    labels += t if train else [IGNORE_INDEX] * len(t)
                eos = getattr(self.tokenizer, "eos_id", None)
                if eos is not None:
                    ids.append(eos)
                    labels.append(eos)
                yield ids, labels
            if not self.config.infinite:
                return

    def _windows(self) -> Iterator[tuple[list[int], list[int], list[int]]]:
        from .loss import IGNORE_INDEX

        W = self.seq_len + 1
        ids, lab, pos = [], [], []
        for s_ids, s_lab in self._samples():
            s_ids, s_lab = s_ids[:W], s_lab[:W]
            if len(ids) + len(s_ids) > W:
                pad = W - len(ids)
                yield ids + [self.config.pad_id] * pad, lab + [IGNORE_INDEX] * pad, pos + list(range(pad))
                ids, lab, pos = [], [], []
            ids += s_ids
            lab += s_lab
            pos += list(range(len(s_ids)))
        if ids:
            pad = W - len(ids)
            yield ids + [self.config.pad_id] * pad, lab + [IGNORE_INDEX] * pad, pos + list(range(pad))

    def __iter__(self):
        batch, skipped = [], 0
        for w in self._windows():
            batch.append(w)
            if len(batch) < self.local_batch_size:
                continue
            ids = torch.tensor([b[0] for b in batch])
            lab = torch.tensor([b[1] for b in batch])
            pos = torch.tensor([b[2] for b in batch])
            batch = []
            if skipped < self.sample_idx:
                skipped += 1
                continue
            self.sample_idx += 1
            skipped += 1
            # input t predicts label t+1
            yield {"input": ids[:, :-1], "positions": pos[:, :-1]}, lab[:, 1:]

    def _local_state(self):
        return {"sample_idx": self.sample_idx}

    def _load_local_state(self, st):
        self.sample_idx = int(st["sample_idx"])
