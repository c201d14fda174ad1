"""Quantized routed experts (parity: reference ``quantization/float8.py``
``Float8GroupedMMConverter`` and the MX grouped-mm path of ``quantization/mx.py``).

MXFP8 on CUDA (expert dims multiples of 128): the forward and data-gradient GEMMs run at FP8
rate on the block-scaled tcgen05 kernel in grouped-rows mode (``ops.grouped._MXGroupedSwiGLU``),
weight gradients in bf16.  Otherwise (CPU, Float8 rowwise, other dims) the expert weights and
routed tokens are quantized to the recipe's codes and dequantized before the bf16 grouped
SwiGLU; gradients pass straight through the quantizers, so the backward GEMMs run on the
quantized forward operands and high-precision output gradients (the "weight gradient in high
precision" variant).
"""
from __future__ import annotations

import os
from dataclasses import dataclass, field
from typing import Any

import torch
import torch.nn as nn

from torchtitan_b200 import ops
from torchtitan_b200.models.common.moe import GroupedExperts
from torchtitan_b200.ops.quant import float8_fake_quant, mx_fake_quant
from torchtitan_b200.protocols.model_converter import ModelConverter
from torchtitan_b200.utils.logging import logger


class _STE(torch.autograd.Function):
    """Forward: quantize-dequantize; backward: identity (straight-through)."""

    @staticmethod
    def forward(ctx, t, fn):
        return fn(t)

    @staticmethod
    def backward(ctx, g):
        return g, None


def _q(t: torch.Tensor, recipe: str, dim: int) -> torch.Tensor:
    if recipe == "mxfp8":
        return _STE.apply(t, lambda x: mx_fake_quant(x, dim))
    return _STE.apply(t, lambda x: float8_fake_quant(x, "rowwise", dim))


class QuantGroupedExperts(GroupedExperts):
    recipe = "mxfp8"

    def forward(self, x: torch.Tensor, counts: torch.Tensor) -> torch.Tensor:
        w1, w2, w3 = self.weights()
        if x.shape[-1] % 32 or w2.shape[-1] % 32:
            return super().forward(x, counts)
        if (self.recipe == "mxfp8" and x.is_cuda and os.environ.get("TTB_MXFP8_KERNEL", "1") != "0"
                and x.shape[-1] % 128 == 0 and w2.shape[-1] % 128 == 0):
            from torchtitan_b200.ops.grouped import mx_grouped_swiglu_cuda

            # FP8-rate grouped GEMMs (block-scaled tcgen05 kernel, grouped-rows mode)
            return mx_grouped_swiglu_cuda(x, w1, w2, w3, counts)
        # w1/w3 [E, H, D] contract over D (last); w2 [E, D, H] contracts over H (last)
        return ops.grouped_swiglu(_q(x, self.recipe, -1), _q(w1, self.recipe, -1), _q(w2, self.recipe, -1),
                                  _q(w3, self.recipe, -1), counts)


class QuantGroupedExpertsConverter(ModelConverter):
    is_quantization = True

    @dataclass(kw_only=True, slots=True)
    class Config(ModelConverter.Config):
        recipe_name: str = "mxfp8"
        """mxfp8 | float8_rowwise"""
        fqns: list[str] = field(default_factory=lambda: ["experts"])

    def convert(self, model: nn.Module) -> None:
        if self.config.recipe_name not in ("mxfp8", "float8_rowwise"):
            raise ValueError(f"unknown grouped recipe {self.config.recipe_name}")
        n = 0
        for fqn, mod in model.named_modules():
            if type(mod) is GroupedExperts and any(f in fqn for f in self.config.fqns):
                mod.__class__ = QuantGroupedExperts
                mod.recipe = self.config.recipe_name
                n += 1
        logger.info(f"quantized grouped experts ({self.config.recipe_name}): {n} modules")

    def post_optimizer_hook(self, model: Any) -> None:
        pass
