"""Model protocol (parity: ``torchtitan/protocols/model.py:13-75``).

``BaseModelArgs`` is the per-family hyper-parameter record: it can be updated
from the trainer config (seq_len, vocab from tokenizer, ...) and reports the
parameter count and training FLOPs per token.  ``BaseModel`` is an
``nn.Module`` that can be built on the meta device and initialised in place
with ``init_weights(buffer_device=...)``.
"""
from __future__ import annotations

import dataclasses
from abc import abstractmethod
from typing import Any

import torch
import torch.nn as nn


@dataclasses.dataclass(kw_only=True)
class BaseModelArgs:
    def update_from_config(self, trainer_config: Any) -> None:
        """Adopt job-level settings (e.g. ``training.seq_len``) before building."""

    def build(self) -> "BaseModel":
        raise NotImplementedError

    def get_nparams_and_flops(self, model: nn.Module, seq_len: int) -> tuple[int, float]:
        raise NotImplementedError

    def to_dict(self) -> dict:
        return dataclasses.asdict(self)


class BaseModel(nn.Module):
    @abstractmethod
    def init_weights(self, buffer_device: torch.device | None = None) -> None:
        ...

    def init_states(self, buffer_device: torch.device | None = None) -> None:
        self.init_weights(buffer_device=buffer_device)

    def verify_module_protocol(self) -> None:
        for name, p in self.named_parameters():
            if p.dtype not in (torch.float32, torch.bfloat16, torch.float16):
                raise TypeError(f"parameter {name} has unsupported dtype {p.dtype}")
