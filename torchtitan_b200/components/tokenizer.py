"""Tokenizers.

``HuggingFaceTokenizer`` loads ``tokenizer.json`` (and optional
``tokenizer_config.json`` for BOS/EOS) from a local assets folder, mirroring
``torchtitan/components/tokenizer.py:98``.  ``SyntheticTokenizer`` needs no
files: it is used with synthetic data, where only ``vocab_size`` matters.
"""
from __future__ import annotations

import json
import os
from abc import ABC, abstractmethod
from dataclasses import dataclass
from typing import Any

from torchtitan_b200.config import Configurable


class BaseTokenizer(ABC, Configurable):
    @dataclass(kw_only=True, slots=True)
    class Config(Configurable.Config):
        pass

    bos_id: int | None = None
    eos_id: int | None = None

    @abstractmethod
    def encode(self, text: str, add_bos: bool = False, add_eos: bool = False) -> list[int]:
        ...

    @abstractmethod
    def decode(self, ids: list[int]) -> str:
        ...

    @abstractmethod
    def get_vocab_size(self) -> int:
        ...


class SyntheticTokenizer(BaseTokenizer):
    @dataclass(kw_only=True, slots=True)
    class Config(BaseTokenizer.Config):
        vocab_size: int = 2048

    def __init__(self, config: Config, tokenizer_path: str | None = None, **kw: Any):
        self.vocab_size = config.vocab_size
        self.bos_id, self.eos_id = 0, 1

    def encode(self, text: str, add_bos: bool = False, add_eos: bool = False) -> list[int]:
        ids = [b % self.vocab_size for b in text.encode()]
        return ([self.bos_id] if add_bos else []) + ids + ([self.eos_id] if add_eos else [])

    def decode(self, ids: list[int]) -> str:
        return bytes(i % 256 for i in ids).decode(errors="replace")

    def get_vocab_size(self) -> int:
        return self.vocab_size


class HuggingFaceTokenizer(BaseTokenizer):
    @dataclass(kw_only=True, slots=True)
    class Config(BaseTokenizer.Config):
        pass

    def __init__(self, config: Config | None = None, tokenizer_path: str = "", **kw: Any):
        from tokenizers import Tokenizer

        path = os.path.join(tokenizer_path, "tokenizer.json")
        if not os.path.exists(path):
            raise FileNotFoundError(f"no tokenizer.json under '{tokenizer_path}'")
        self.tok = Tokenizer.from_file(path)
        self.bos_token = self.eos_token = None
        self.chat_template: str | None = None
        cfg_path = os.path.join(tokenizer_path, "tokenizer_config.json")
        if os.path.exists(cfg_path):
            with open(cfg_path) as f:
                tc = json.load(f)

            def _tok(v):
                return v.get("content") if isinstance(v, dict) else v

            self.bos_token, self.eos_token = _tok(tc.get("bos_token")), _tok(tc.get("eos_token"))
            self.chat_template = tc.get("chat_template")
        vocab = self.tok.get_vocab(with_added_tokens=True)
        for cand in (self.bos_token, "<|begin_of_text|>", "<s>", "[BOS]"):
            if cand and cand in vocab:
                self.bos_id = vocab[cand]
                break
        for cand in (self.eos_token, "<|end_of_text|>", "</s>", "[EOS]"):
            if cand and cand in vocab:
                self.eos_id = vocab[cand]
                break

    def encode(self, text: str, add_bos: bool = False, add_eos: bool = False) -> list[int]:
        ids = self.tok.encode(text, add_special_tokens=False).ids
        if add_bos and self.bos_id is not None:
            ids = [self.bos_id] + ids
        if add_eos and self.eos_id is not None:
            ids = ids + [self.eos_id]
        return ids

    def decode(self, ids: list[int]) -> str:
        return self.tok.decode(ids)

    def get_vocab_size(self) -> int:
        return self.tok.get_vocab_size(with_added_tokens=True)

    def apply_chat_template(self, messages: list[dict], add_generation_prompt: bool = False) -> list[int]:
        """Render ``messages`` with the tokenizer's own chat template (jinja) and encode them."""
        if not self.chat_template:
            raise ValueError("this tokenizer has no chat_template")
        import jinja2

        text = jinja2.Template(self.chat_template).render(
            messages=messages, add_generation_prompt=add_generation_prompt, bos_token=self.bos_token or "",
            eos_token=self.eos_token or "")
        return self.encode(text)
