"""Grouped SwiGLU experts: out_r = w2[e] (silu(w1[e] x_r) * w3[e] x_r) for rows r of expert e.

On CUDA the three GEMMs run as grouped tcgen05 GEMMs over expert segments
(``ops/grouped.py`` on ``csrc/gemm_tcgen05.cu``); on CPU a per-expert loop.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def _reference(x, w1, w2, w3, counts):
    outs = []
    start = 0
    for e, n in enumerate(counts.tolist()):
        xe = x[start:start + n]
        outs.append((F.silu(xe @ w1[e].t()) * (xe @ w3[e].t())) @ w2[e].t())
        start += n
    return torch.cat(outs, 0) if outs else x.new_zeros(0, w2.shape[1])


def grouped_swiglu(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor, w3: torch.Tensor,
                   counts: torch.Tensor) -> torch.Tensor:
    if not x.is_cuda:
        return _reference(x, w1, w2, w3, counts)
    from .grouped import grouped_swiglu_cuda

    return grouped_swiglu_cuda(x, w1, w2, w3, counts)
