"""Token-sum cross entropy (parity: ``torchtitan/components/loss.py:16-53``).

The loss is a SUM over non-ignored tokens in fp32; the trainer divides by the
global valid-token count so gradient accumulation and DP are exact.  On CUDA
the sum is computed by the fused online-softmax kernel
(``ops.cross_entropy_sum``) which never materialises fp32 logits.
"""
from __future__ import annotations

from collections.abc import Callable
from typing import Any, TypeAlias

import torch

from torchtitan_b200 import ops

IGNORE_INDEX = -100
LossFunction: TypeAlias = Callable[..., torch.Tensor]


def cross_entropy_loss(pred: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
    return ops.cross_entropy_sum(pred.flatten(0, -2), labels.flatten(), ignore_index=IGNORE_INDEX)


def build_cross_entropy_loss(compile_config: Any = None, **kwargs: Any) -> LossFunction:
    return cross_entropy_loss


def mse_loss(pred: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
    return torch.nn.functional.mse_loss(pred.float(), labels.float().detach(), reduction="sum")


def build_mse_loss(compile_config: Any = None, **kwargs: Any) -> LossFunction:
    return mse_loss
