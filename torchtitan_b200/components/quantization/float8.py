"""Float8 training converter (parity: reference ``quantization/float8.py:1-310``:
tensorwise, rowwise and rowwise_with_gw_hp recipes on linear layers)."""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any

import torch
import torch.nn as nn

from torchtitan_b200 import ops
from torchtitan_b200.models.common import Linear
from torchtitan_b200.models.common.layers import _local
from torchtitan_b200.ops.quant import float8_fake_quant
from torchtitan_b200.protocols.model_converter import ModelConverter
from torchtitan_b200.utils.logging import logger

from .utils import swap_linears


def _kernel_path(x: torch.Tensor) -> bool:
    """E4M3 GEMMs on the tensor cores (``gemm_f8``: the block-scaled tcgen05 kernel with unit
    block scales and the fp32 row / tensor scales applied in its epilogue); ``TTB_FLOAT8_KERNEL=0``
    selects the quantize-dequantize emulation on the bf16 GEMM."""
    import os

    return x.is_cuda and os.environ.get("TTB_FLOAT8_KERNEL", "1") != "0"


def _f8_mm(a: torch.Tensor, b: torch.Tensor, rowwise: bool) -> torch.Tensor:
    """``a @ b.T`` with both operands quantized along the contraction (last) dimension."""
    from torchtitan_b200.ops._ext import ext

    qa, ia = ext().f8_quantize(a.contiguous(), rowwise)
    qb, ib = ext().f8_quantize(b.contiguous(), rowwise)
    return ext().gemm_f8(qa, ia, qb, ib)


class _F8LinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, recipe):
        ctx.save_for_backward(x, w)
        ctx.recipe = recipe
        g = "tensorwise" if recipe == "tensorwise" else "rowwise"
        if _kernel_path(x) and x.dtype == torch.bfloat16:
            x2 = x.reshape(-1, x.shape[-1])
            return _f8_mm(x2, w.to(x.dtype), g == "rowwise").view(*x.shape[:-1], w.shape[0])
        return ops.linear(float8_fake_quant(x, g, -1), float8_fake_quant(w, g, -1))

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        r = ctx.recipe
        g = "tensorwise" if r == "tensorwise" else "rowwise"
        x2, dy2 = x.reshape(-1, x.shape[-1]), dy.reshape(-1, dy.shape[-1])
        if _kernel_path(x) and x.dtype == torch.bfloat16:
            rw = g == "rowwise"
            wb = w.to(x.dtype)
            dx = _f8_mm(dy2.to(x.dtype), wb.t(), rw).view(x.shape)
            if r == "rowwise_with_gw_hp":
                dw = ops.matmul(dy2.t().contiguous(), x2)
            else:
                dw = _f8_mm(dy2.to(x.dtype).t(), x2.t(), rw)
            return dx, dw.to(w.dtype), None
        dx = ops.matmul(float8_fake_quant(dy2, g, -1), float8_fake_quant(w, g, 0)).view(x.shape)
        if r == "rowwise_with_gw_hp":  # weight gradient kept in high precision
            dw = ops.matmul(dy2.t().contiguous(), x2)
        else:
            dw = ops.matmul(float8_fake_quant(dy2, g, 0).t().contiguous(), float8_fake_quant(x2, g, 0))
        return dx, dw.to(w.dtype), None


class Float8Linear(Linear):
    recipe = "tensorwise"

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        w = _local(self.weight)

        def mm(a, b):
            return _F8LinearFn.apply(a, b.to(a.dtype), self.recipe)

        if self.tp_mode is None:
            y = mm(x, w)
        else:
            from torchtitan_b200.parallel import tensor_parallel as tp

            y = tp.tp_linear(x, w, self.tp_mode, self.tp_group, self.sequence_parallel, matmul=mm)
        return y if self.bias is None else y + _local(self.bias).to(y.dtype)


class Float8LinearConverter(ModelConverter):
    is_quantization = True

    @dataclass(kw_only=True, slots=True)
    class Config(ModelConverter.Config):
        recipe_name: str = "tensorwise"
        """tensorwise | rowwise | rowwise_with_gw_hp"""
        filter_fqns: list[str] = field(default_factory=lambda: ["output"])
        enable_fsdp_float8_all_gather: bool = False
        precompute_float8_dynamic_scale_for_fsdp: bool = False

    def __init__(self, config: Config, **kw: Any):
        super().__init__(config, **kw)
        if config.recipe_name not in ("tensorwise", "rowwise", "rowwise_with_gw_hp"):
            raise ValueError(f"unknown Float8 recipe {config.recipe_name}")

    def convert(self, model: nn.Module) -> None:
        n = swap_linears(model, Float8Linear, 16, self.config.filter_fqns, recipe=self.config.recipe_name)
        logger.info(f"Float8: swapped {n} linear layers ({self.config.recipe_name})")
