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


# ------------------------------------------------------- deterministic dispatch / combine
class _Dispatch(torch.autograd.Function):
    """routed[r] = x[token_of[r]] (row gather); backward: per-token sum over its slots
    (``moe_combine_fwd`` without gates), a gather-sum in a fixed order instead of atomics."""

    @staticmethod
    def forward(ctx, x, token_of, pos):
        from ._ext import ext

        ctx.save_for_backward(pos)
        return ext().gather_rows(x.contiguous(), token_of)

    @staticmethod
    def backward(ctx, g):
        from ._ext import ext

        (pos,) = ctx.saved_tensors
        return ext().moe_combine_fwd(None, g.contiguous(), pos, None), None, None


class _Combine(torch.autograd.Function):
    """out[t] = base[t] + sum_j w[t, j] * y[pos[t, j]] (fp32 accumulation); backward by gathers
    and per-slot dot products."""

    @staticmethod
    def forward(ctx, base, y, w, pos, token_of, order):
        from ._ext import ext

        wf = None if w is None else w.float().contiguous()
        y = y.contiguous()
        ctx.save_for_backward(y, wf, pos, token_of, order)
        ctx.has_base, ctx.has_w = base is not None, w is not None
        ctx.w_dtype = None if w is None else w.dtype
        return ext().moe_combine_fwd(None if base is None else base.contiguous(), y, pos, wf)

    @staticmethod
    def backward(ctx, dout):
        from ._ext import ext

        y, wf, pos, token_of, order = ctx.saved_tensors
        dout = dout.contiguous()
        scale = None if wf is None else wf.reshape(-1)[order].contiguous()
        need_dw = bool(ctx.has_w and ctx.needs_input_grad[2])
        dy, dw = ext().moe_combine_bwd(dout, y, pos, token_of, scale, need_dw)
        return (dout if ctx.has_base else None), dy, (dw.to(ctx.w_dtype) if need_dw else None), None, None, None


def combine_kernel_enabled(x: torch.Tensor) -> bool:
    """The deterministic dispatch/combine kernels (``csrc/moe_combine.cu``) on CUDA bf16 rows;
    ``TTB_MOE_COMBINE_KERNEL=0`` selects the PyTorch index ops."""
    import os

    return (x.is_cuda and x.dtype == torch.bfloat16 and x.shape[-1] % 8 == 0
            and os.environ.get("TTB_MOE_COMBINE_KERNEL", "1") != "0")


def slot_positions(order: torch.Tensor, top_k: int) -> torch.Tensor:
    """pos[t, j]: the expert-sorted row that holds slot j of token t (inverse of ``order``)."""
    inv = torch.empty_like(order)
    inv[order] = torch.arange(order.numel(), device=order.device)
    return inv.view(-1, top_k)


def moe_dispatch(x: torch.Tensor, token_of: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
    return _Dispatch.apply(x, token_of, pos)


def moe_combine(base, y, w, pos, token_of, order) -> torch.Tensor:
    return _Combine.apply(base, y, w, pos, token_of, order)
