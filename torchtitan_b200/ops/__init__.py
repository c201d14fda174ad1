"""Hot ops with autograd.  CUDA tensors run the sm_100a kernels in
``torchtitan_b200/csrc`` (loaded from the in-tree ``_C`` extension, no
fallback); CPU tensors run ``ops.reference``.

Public functions:
  linear(x, w)                       y = x @ w.T           (tcgen05 GEMM)
  matmul(a, b)                       a @ b                 (tcgen05 GEMM)
  rms_norm(x, w, eps)                                        (fused fwd/bwd)
  rope(x, cos, sin)                  interleaved-pair rotary embedding
  swiglu(a, b)                       silu(a) * b
  attention(q, k, v, causal, scale)  flash attention, GQA, [B,S,H,D]
  cross_entropy_sum(logits, labels)  fp32 sum over valid tokens
  fused_adamw_(...)                  multi-tensor AdamW step
"""
from __future__ import annotations

import torch

from . import reference as _ref
from ._ext import available, ext

__all__ = [
    "available", "linear", "matmul", "rms_norm", "rope", "swiglu", "attention",
    "cross_entropy_sum", "fused_adamw_",
]


def _cuda(*ts) -> bool:
    return any(t.is_cuda for t in ts if torch.is_tensor(t))


# --------------------------------------------------------------------------- GEMM
from .gemm import linear, matmul  # noqa: E402
from .attention import attention  # noqa: E402


# ------------------------------------------------------------------------ RMSNorm
class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps):
        shp = x.shape
        x2 = x.reshape(-1, shp[-1])
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        y, rstd = ext().rmsnorm_fwd(x2, w, eps)
        ctx.save_for_backward(x2, w, rstd)
        return y.view(shp)

    @staticmethod
    def backward(ctx, dy):
        x2, w, rstd = ctx.saved_tensors
        dx, dw = ext().rmsnorm_bwd(dy.reshape(x2.shape).contiguous(), x2, w, rstd)
        return dx.view(dy.shape), dw.to(w.dtype), None


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    if not _cuda(x):
        return _ref.rms_norm(x, w, eps)
    return _RMSNorm.apply(x, w, eps)


# --------------------------------------------------------------------------- RoPE
class _Rope(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, cos, sin):
        ctx.save_for_backward(cos, sin)
        return ext().rope(x.contiguous(), cos, sin, False)

    @staticmethod
    def backward(ctx, dy):
        cos, sin = ctx.saved_tensors
        return ext().rope(dy.contiguous(), cos, sin, True), None, None


def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x: [B,S,H,D]; cos/sin: [S, D/2] fp32 (position-major), or [B, S, D/2] for per-row
    positions (packed documents, multimodal 3-D positions)."""
    if not _cuda(x):
        return _ref.rope(x, cos, sin)
    return _Rope.apply(x, cos, sin)


# ------------------------------------------------------------------------- SwiGLU
class _SwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a, b):
        a, b = a.contiguous(), b.contiguous()
        ctx.save_for_backward(a, b)
        return ext().swiglu_fwd(a, b)

    @staticmethod
    def backward(ctx, dy):
        a, b = ctx.saved_tensors
        da, db = ext().swiglu_bwd(dy.contiguous(), a, b)
        return da, db


def swiglu(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    if not _cuda(a):
        return _ref.swiglu(a, b)
    return _SwiGLU.apply(a, b)


# ------------------------------------------------------------------ cross entropy
class _CESum(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, labels, ignore_index):
        logits = logits.contiguous()
        loss, lse = ext().ce_fwd(logits, labels.contiguous(), ignore_index)
        ctx.save_for_backward(logits, labels, lse)
        ctx.ignore_index = ignore_index
        return loss

    @staticmethod
    def backward(ctx, g):
        logits, labels, lse = ctx.saved_tensors
        dlogits = ext().ce_bwd(logits, labels, lse, g.float().reshape(1).contiguous(), ctx.ignore_index)
        return dlogits, None, None


def cross_entropy_sum(logits: torch.Tensor, labels: torch.Tensor, ignore_index: int = -100) -> torch.Tensor:
    if type(logits).__name__ == "DTensor" or not _cuda(logits):
        return _ref.cross_entropy_sum(logits, labels, ignore_index)
    return _CESum.apply(logits, labels, ignore_index)


# ---------------------------------------------------------------- MoE experts
from .moe import combine_kernel_enabled, grouped_swiglu, moe_combine, moe_dispatch, slot_positions  # noqa: E402
from .grouped import grouped_swiglu_padded  # noqa: E402
from .attention import attention_with_lse, document_attention  # noqa: E402


# -------------------------------------------------------------------------- AdamW
def fused_adamw_(params, grads, exp_avgs, exp_avg_sqs, *, lr: float, beta1: float, beta2: float,
                 eps: float, weight_decay: float, step: int, copies=None, clip_total=None,
                 clip_max: float = 0.0) -> None:
    """``copies``: optional bf16 tensors receiving the updated fp32 params (compute weights).
    ``clip_total``: optional device scalar (sum of squared grad norms); grads are scaled by
    min(1, clip_max / (sqrt(clip_total) + 1e-6)) inside the kernel."""
    if not params:
        return
    if not params[0].is_cuda:
        if clip_total is not None:
            coef = float(torch.clamp(clip_max / (clip_total.sqrt() + 1e-6), max=1.0))
            grads = [g * coef for g in grads]
        _ref.adamw_(params, grads, exp_avgs, exp_avg_sqs, lr=lr, beta1=beta1, beta2=beta2, eps=eps,
                    weight_decay=weight_decay, step=step)
        for p, c in zip(params, copies or []):
            if c is not None:
                c.copy_(p)
        return
    cp = [c if c is not None else torch.empty(0, device=params[0].device) for c in (copies or [])]
    ext().adamw(list(params), list(grads), list(exp_avgs), list(exp_avg_sqs), float(lr), float(beta1),
                float(beta2), float(eps), float(weight_decay), int(step), cp,
                clip_total.float().reshape(()).contiguous() if clip_total is not None else None, float(clip_max))
