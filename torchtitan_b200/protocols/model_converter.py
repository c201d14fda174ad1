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


def _named_converter(name: str) -> Any:
    from torchtitan_b200.components.quantization import Float8LinearConverter, MXFP8Converter

    if name in ("mx", "mxfp8"):
        return MXFP8Converter.Config()
    if name in ("mxfp8_grouped", "float8_rowwise_grouped"):
        from torchtitan_b200.components.quantization.grouped import QuantGroupedExpertsConverter

        return QuantGroupedExpertsConverter.Config(recipe_name=name[: -len("_grouped")])
    if name.startswith("float8"):
        recipe = name[len("float8_"):] if name != "float8" else "tensorwise"
        return Float8LinearConverter.Config(recipe_name=recipe)
    raise ValueError(f"unknown model converter '{name}'")


class ModelConvertersContainer(Configurable):
    @dataclass(kw_only=True, slots=True)
    class Config(Configurable.Config):
        converters: list[Any] = field(default_factory=list)
        names: list[str] = field(default_factory=list)
        """Shortcut for the command line: ``mxfp8``, ``float8``, ``float8_rowwise``,
        ``float8_rowwise_with_gw_hp`` for linears; ``mxfp8_grouped``, ``float8_rowwise_grouped``
        for routed experts (default settings of each converter)."""

    def __init__(self, config: Config, **kwargs: Any):
        cfgs = list(config.converters) + [_named_converter(n) for n in config.names]
        self.converters = [c.build(**kwargs) for c in cfgs]
        nq = sum(1 for c in self.converters if getattr(c, "is_quantization", False)
                 and type(c).__name__ != "QuantGroupedExpertsConverter")
        if nq > 1:
            raise ValueError("at most one quantization converter may be configured")

    def convert(self, model: nn.Module) -> None:
        for c in self.converters:
            c.convert(model)

    def post_optimizer_hook(self, model: nn.Module | list[nn.Module]) -> None:
        for c in self.converters:
            c.post_optimizer_hook(model)
