"""Parameter-holding building blocks that route compute through ``ops``.

``Linear`` owns only ``weight`` ([out, in], no bias, as in the reference
Llama/Kimi layers).  Tensor parallelism is a property of the layer, set by
the parallelize functions: ``tp_mode`` is ``None``, ``"col"`` or ``"row"``
and the layer issues its own collectives (sequence all-gather before a
column-parallel GEMM, reduce-scatter after a row-parallel one) through
``parallel.tensor_parallel``.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn

from torchtitan_b200 import ops


def _local(t: torch.Tensor) -> torch.Tensor:
    return t.to_local() if type(t).__name__ == "DTensor" else t


def compute_ffn_hidden_dim(dim: int, multiple_of: int = 256, ffn_dim_multiplier: float | None = None) -> int:
    hidden = int(2 * (4 * dim) / 3)
    if ffn_dim_multiplier is not None:
        hidden = int(ffn_dim_multiplier * hidden)
    return multiple_of * ((hidden + multiple_of - 1) // multiple_of)


class Linear(nn.Module):
    def __init__(self, in_features: int, out_features: int, init_std: float = 0.02, bias: bool = False):
        super().__init__()
        self.in_features, self.out_features = in_features, out_features
        self.weight = nn.Parameter(torch.empty(out_features, in_features))
        self.bias = nn.Parameter(torch.empty(out_features)) if bias else None
        self.init_std = init_std
        self.init_cutoff: float | None = None
        self.tp_mode: str | None = None
        self.tp_group = None
        self.sequence_parallel = False

    def init_weights(self, std: float | None = None) -> None:
        s = self.init_std if std is None else std
        c = self.init_cutoff if self.init_cutoff is not None else 2.0
        nn.init.trunc_normal_(self.weight, mean=0.0, std=s, a=-c, b=c)
        if self.bias is not None:
            nn.init.zeros_(self.bias)

    grad_reduce_group = None  # replicated over TP on sequence-sharded inputs: reduce weight grads

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        w = _local(self.weight)
        if self.grad_reduce_group is not None:
            from torchtitan_b200.parallel.tensor_parallel import grad_all_reduce

            w = grad_all_reduce(w, self.grad_reduce_group)
        if self.tp_mode is None:
            y = ops.linear(x, w)
        else:
            from torchtitan_b200.parallel import tensor_parallel as tp

            y = tp.tp_linear(x, w, self.tp_mode, self.tp_group, self.sequence_parallel)
        if self.bias is not None:
            b = _local(self.bias)
            g = self.bias_grad_reduce_group or self.grad_reduce_group
            if g is not None:
                from torchtitan_b200.parallel.tensor_parallel import grad_all_reduce

                b = grad_all_reduce(b, g)
            y = y + b.to(y.dtype)
        return y

    bias_grad_reduce_group = None  # replicated bias of a row-parallel layer on sequence shards

    def extra_repr(self) -> str:
        return f"in={self.in_features}, out={self.out_features}, tp={self.tp_mode}"


class Embedding(nn.Module):
    def __init__(self, num_embeddings: int, embedding_dim: int, init_std: float = 1.0):
        super().__init__()
        self.num_embeddings, self.embedding_dim = num_embeddings, embedding_dim
        self.weight = nn.Parameter(torch.empty(num_embeddings, embedding_dim))
        self.init_std = init_std

    def init_weights(self) -> None:
        nn.init.normal_(self.weight, std=self.init_std)

    def forward(self, tokens: torch.Tensor) -> torch.Tensor:
        return nn.functional.embedding(tokens, _local(self.weight))


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float = 1e-5):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.empty(dim))

    def init_weights(self) -> None:
        nn.init.ones_(self.weight)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        w = _local(self.weight)
        return ops.rms_norm(x, w.to(x.dtype) if w.dtype != x.dtype else w, self.eps)


class FeedForward(nn.Module):
    """SwiGLU MLP: ``w2(silu(w1 x) * w3 x)``."""

    def __init__(self, dim: int, hidden_dim: int):
        super().__init__()
        self.w1 = Linear(dim, hidden_dim)
        self.w2 = Linear(hidden_dim, dim)
        self.w3 = Linear(dim, hidden_dim)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.w2(ops.swiglu(self.w1(x), self.w3(x)))

    def init_weights(self, init_std: float) -> None:
        self.w1.init_weights(0.02)
        self.w2.init_weights(init_std)
        self.w3.init_weights(init_std)


def depth_init_std(layer_id: int, n_layers: int, depth_init: bool = True) -> float:
    return 0.02 / math.sqrt(2 * (layer_id + 1)) if depth_init else 0.02 / math.sqrt(2 * n_layers)
