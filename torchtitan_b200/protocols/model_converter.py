"""Sequential model converters (e.g. MXFP8 linear swap).

Parity: ``torchtitan/protocols/model_converter.py:17-101`` -- converters run in
order on the meta-device model, at most one quantization converter is allowed,
and a post-optimizer hook is forwarded to each.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any

import torch.nn as nn

from torchtitan_b200.config import Configurable


class ModelConverter(Configurable):
    is_quantization: bool = False

    @dataclass(kw_only=True, slots=True)
    class Config(Configurable.Config):
        pass

    def __init__(self, config: Config, **kwargs: Any):
        self.config = config

    def convert(self, model: nn.Module) -> None:
        raise NotImplementedError

    def post_optimizer_hook(self, model: nn.Module | list[nn.Module]) -> None:
        pass


class ModelConvertersContainer(Configurable):
    @dataclass(kw_only=True, slots=True)
    class Config(Configurable.Config):
        converters: list[Any] = field(default_factory=list)

    def __init__(self, config: Config, **kwargs: Any):
        self.converters = [c.build(**kwargs) for c in config.converters]
        nq = sum(1 for c in self.converters if getattr(c, "is_quantization", False))
        if nq > 1:
            raise ValueError("at most one quantization converter may be configured")

    def convert(self, model: nn.Module) -> None:
        for c in self.converters:
            c.convert(model)

    def post_optimizer_hook(self, model: nn.Module | list[nn.Module]) -> None:
        for c in self.converters:
            c.post_optimizer_hook(model)
