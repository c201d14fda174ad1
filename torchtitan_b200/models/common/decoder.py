"""Decoder-only LM skeleton shared by the model families
(parity: ``models/common/decoder.py:38-198``).

FQNs: ``tok_embeddings.weight``, ``layers.<i>.*``, ``norm.weight``,
``output.weight``.  Layers live in an ``nn.ModuleDict`` keyed by the string
layer index so pipeline stages can delete layers and keep FQNs stable.
Any of ``tok_embeddings``/``norm``/``output`` may be ``None`` on a pipeline
stage that does not own it.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from torchtitan_b200.protocols import BaseModel


class Decoder(BaseModel):
    rope: nn.Module

    def _rope_tables(self, seq_len: int, positions: torch.Tensor | None):
        cos, sin = self.rope.tables(seq_len, positions)
        return cos, sin

    def forward(self, tokens: torch.Tensor, attention_masks=None, positions: torch.Tensor | None = None):
        h = self.tok_embeddings(tokens) if self.tok_embeddings is not None else tokens
        # under sequence parallelism h holds this rank's sequence shard; attention sees the full sequence
        seq = tokens.shape[1] if self.tok_embeddings is not None else h.shape[1] * getattr(self, "_sp_degree", 1)
        cos, sin = self._rope_tables(seq, positions)
        for layer in self.layers.values():
            h = layer(h, cos, sin, attention_masks)
        h = self.norm(h) if self.norm is not None else h
        return self.output(h) if self.output is not None else h
