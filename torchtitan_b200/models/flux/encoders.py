"""Frozen text encoders and tokenizers of FLUX (behaviour parity: reference
``models/flux/model/hf_embedder.py`` and ``models/flux/tokenizer.py``): T5 (per-token
states, ``[B, max_t5_len, d_model]``) and CLIP-L (pooled, ``[B, 768]``), both Hugging
Face ``transformers`` models loaded from local directories.

Without local weights (``random_init``) the encoders are built from small
configurations of the right output widths with random weights, and the tokenizers
hash characters into the vocabulary: enough for synthetic runs and tests, never for
a real model.
"""
from __future__ import annotations

import os
from dataclasses import dataclass

import torch
import torch.nn as nn


@dataclass(kw_only=True, slots=True)
class FluxEncoderConfig:
    t5_encoder: str = "google/t5-v1_1-xxl"
    """Local directory of the T5 encoder (and its tokenizer)."""
    clip_encoder: str = "openai/clip-vit-large-patch14"
    """Local directory of the CLIP text encoder (and its tokenizer)."""
    autoencoder_path: str = "assets/hf/FLUX.1-dev/ae.safetensors"
    max_t5_encoding_len: int = 256
    random_init: bool = True
    """Build random-weight encoders when the directories do not exist (synthetic runs)."""


class _HashTokenizer:
    """Characters hashed into ``vocab`` ids, padded/truncated to ``length``."""

    def __init__(self, vocab: int, length: int):
        self.vocab, self.length = vocab, length

    def __call__(self, texts: list[str]) -> torch.Tensor:
        out = torch.zeros(len(texts), self.length, dtype=torch.long)
        for i, t in enumerate(texts):
            ids = [(ord(ch) * 2654435761) % (self.vocab - 2) + 2 for ch in t][: self.length - 1] + [1]
            out[i, : len(ids)] = torch.tensor(ids)
        return out


class FluxTextEncoders(nn.Module):
    def __init__(self, cfg: FluxEncoderConfig, context_dim: int, vec_dim: int):
        super().__init__()
        import transformers

        self.max_len = cfg.max_t5_encoding_len
        if os.path.isdir(cfg.t5_encoder):
            self.t5 = transformers.T5EncoderModel.from_pretrained(cfg.t5_encoder)
            tok = transformers.AutoTokenizer.from_pretrained(cfg.t5_encoder)
            self.t5_tok = lambda texts: tok(texts, padding="max_length", truncation=True, max_length=self.max_len,
                                            return_tensors="pt").input_ids
        elif cfg.random_init:
            tc = transformers.T5Config(vocab_size=512, d_model=context_dim, d_kv=32, d_ff=256, num_layers=1,
                                       num_heads=2, feed_forward_proj="gated-gelu")
            self.t5 = transformers.T5EncoderModel(tc)
            self.t5_tok = _HashTokenizer(512, self.max_len)
        else:
            raise FileNotFoundError(f"T5 encoder directory {cfg.t5_encoder} not found")
        if os.path.isdir(cfg.clip_encoder):
            self.clip = transformers.CLIPTextModel.from_pretrained(cfg.clip_encoder)
            ctok = transformers.AutoTokenizer.from_pretrained(cfg.clip_encoder)
            self.clip_tok = lambda texts: ctok(texts, padding="max_length", truncation=True, max_length=77,
                                               return_tensors="pt").input_ids
        elif cfg.random_init:
            cc = transformers.CLIPTextConfig(vocab_size=512, hidden_size=vec_dim, intermediate_size=128,
                                             num_hidden_layers=1, num_attention_heads=2, max_position_embeddings=77,
                                             eos_token_id=1)
            self.clip = transformers.CLIPTextModel(cc)
            self.clip_tok = _HashTokenizer(512, 77)
        else:
            raise FileNotFoundError(f"CLIP encoder directory {cfg.clip_encoder} not found")
        self.requires_grad_(False)
        self.eval()

    def tokenize(self, texts: list[str]) -> dict[str, torch.Tensor]:
        return {"t5_tokens": self.t5_tok(texts), "clip_tokens": self.clip_tok(texts)}

    @torch.no_grad()
    def forward(self, t5_tokens: torch.Tensor, clip_tokens: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        txt = self.t5(input_ids=t5_tokens).last_hidden_state
        vec = self.clip(input_ids=clip_tokens).pooler_output
        return txt, vec
