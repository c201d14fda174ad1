"""Model registration record (parity: ``torchtitan/protocols/model_spec.py:29-51``)."""
from __future__ import annotations

from collections.abc import Callable
from dataclasses import dataclass
from typing import Any

from .model import BaseModelArgs


@dataclass
class ModelSpec:
    name: str
    flavor: str
    model: BaseModelArgs
    parallelize_fn: Callable[..., Any]
    pipelining_fn: Callable[..., Any] | None
    build_loss_fn: Callable[..., Any]
    post_optimizer_build_fn: Callable[..., Any] | None = None
    state_dict_adapter: type | None = None
