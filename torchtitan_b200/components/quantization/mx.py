"""MXFP8 training converter (parity: reference ``quantization/mx.py:25-134``:
MXFP8 1x32 E8M0 blocks with RCEIL scale rounding on linear layers matched by FQN)."""
from __future__ import annotations

import os
from dataclasses import dataclass, field
from typing import Any

import torch
import torch.nn as nn

from torchtitan_b200 import ops
from torchtitan_b200.models.common import Linear
from torchtitan_b200.models.common.layers import _local
from torchtitan_b200.ops.quant import mx_fake_quant
from torchtitan_b200.protocols.model_converter import ModelConverter
from torchtitan_b200.utils.logging import logger

from .utils import swap_linears


def _use_block_scaled_kernel(t: torch.Tensor) -> bool:
    # the tcgen05 block-scaled GEMM (TTB_MXFP8_KERNEL=0 multiplies the same quantized values
    # on the bf16 GEMM instead)
    return t.is_cuda and os.environ.get("TTB_MXFP8_KERNEL", "1") != "0"


class _MXLinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w):
        ctx.save_for_backward(x, w)
        if _use_block_scaled_kernel(x):
            from torchtitan_b200.ops.mx_gemm import mx_linear

            return mx_linear(x, w).to(x.dtype)
        return ops.linear(mx_fake_quant(x, -1), mx_fake_quant(w, -1))

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        x2, dy2 = x.reshape(-1, x.shape[-1]), dy.reshape(-1, dy.shape[-1])
        if _use_block_scaled_kernel(dy):
            from torchtitan_b200.ops.mx_gemm import mx_linear

            # every operand quantized along its GEMM's contraction dimension
            dx = mx_linear(dy2.contiguous(), w.t().contiguous()).view(x.shape).to(x.dtype)
            dw = mx_linear(dy2.t().contiguous(), x2.t().contiguous()).to(w.dtype)
            return dx, dw
        # dgrad: contraction over `out` -> dy blocked along its last dim, W blocked along dim 0
        dx = ops.matmul(mx_fake_quant(dy2, -1), mx_fake_quant(w, 0)).view(x.shape)
        # wgrad: contraction over tokens -> both blocked along dim 0
        dw = ops.matmul(mx_fake_quant(dy2, 0).t(), mx_fake_quant(x2, 0)).to(w.dtype)
        return dx, dw


class MXFP8Linear(Linear):
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        w = _local(self.weight)

        def mm(a, b):
            if a.shape[:-1].numel() % 32:
                return ops.linear(a, b)  # wgrad blocks need tokens in multiples of 32
            return _MXLinearFn.apply(a, b.to(a.dtype))

        if self.tp_mode is None:
            y = mm(x, w)
        else:
            from torchtitan_b200.parallel import tensor_parallel as tp

            y = tp.tp_linear(x, w, self.tp_mode, self.tp_group, self.sequence_parallel, matmul=mm)
        return y if self.bias is None else y + _local(self.bias).to(y.dtype)


class MXFP8Converter(ModelConverter):
    is_quantization = True

    @dataclass(kw_only=True, slots=True)
    class Config(ModelConverter.Config):
        recipe_name: str = "mxfp8_rceil"
        filter_fqns: list[str] = field(default_factory=lambda: ["output"])

    def __init__(self, config: Config, **kw: Any):
        super().__init__(config, **kw)
        if config.recipe_name not in ("mxfp8_rceil", "mxfp8_cublas_rceil", "mxfp8"):
            raise ValueError(f"unknown MX recipe {config.recipe_name}")

    def convert(self, model: nn.Module) -> None:
        n = swap_linears(model, MXFP8Linear, 32, self.config.filter_fqns)
        logger.info(f"MXFP8: swapped {n} linear layers ({self.config.recipe_name})")
