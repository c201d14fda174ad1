"""Plain-PyTorch fp32 restatements of every kernel in ``csrc/``.

They are the CPU execution path and the numerics oracle for the CUDA tests.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (y * w.float()).to(x.dtype)


def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x: [B,S,H,D] with interleaved (re, im) pairs; cos/sin: [S, D/2] or per-row [B, S, D/2]."""
    xf = x.float().unflatten(-1, (-1, 2))
    re, im = xf[..., 0], xf[..., 1]
    c = (cos[:, :, None, :] if cos.dim() == 3 else cos[None, :, None, :]).float()
    s = (sin[:, :, None, :] if sin.dim() == 3 else sin[None, :, None, :]).float()
    out = torch.stack([re * c - im * s, re * s + im * c], -1).flatten(-2)
    return out.to(x.dtype)


def swiglu(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    return (F.silu(a.float()) * b.float()).to(a.dtype)


def attention(q, k, v, causal: bool = True, scale: float | None = None):
    """q [B,S,H,D], k/v [B,S,Hkv,Dv] -> [B,S,H,Dv] (GQA by head grouping)."""
    H, Hk = q.shape[2], k.shape[2]
    if Hk != H:
        k = k.repeat_interleave(H // Hk, dim=2)
        v = v.repeat_interleave(H // Hk, dim=2)
    scale = scale if scale is not None else 1.0 / math.sqrt(q.shape[-1])
    Sq, Sk = q.shape[1], k.shape[1]
    mask = None
    if causal:  # bottom-right aligned: query i sees keys j <= i + (Sk - Sq)
        mask = torch.ones(Sq, Sk, dtype=torch.bool, device=q.device).tril(diagonal=Sk - Sq)
    o = F.scaled_dot_product_attention(q.transpose(1, 2).float(), k.transpose(1, 2).float(),
                                       v.transpose(1, 2).float(), attn_mask=mask, scale=scale)
    return o.transpose(1, 2).to(q.dtype)


def cross_entropy_sum(logits: torch.Tensor, labels: torch.Tensor, ignore_index: int = -100) -> torch.Tensor:
    return F.cross_entropy(logits.float(), labels, reduction="sum", ignore_index=ignore_index)


def adamw_(params, grads, exp_avgs, exp_avg_sqs, *, lr, beta1, beta2, eps, weight_decay, step):
    bc1 = 1 - beta1 ** step
    bc2 = 1 - beta2 ** step
    for p, g, m, v in zip(params, grads, exp_avgs, exp_avg_sqs):
        gf = g.float()
        m.mul_(beta1).add_(gf, alpha=1 - beta1)
        v.mul_(beta2).addcmul_(gf, gf, value=1 - beta2)
        p.mul_(1 - lr * weight_decay)
        denom = (v / bc2).sqrt_().add_(eps)
        p.addcdiv_(m, denom, value=-lr / bc1)
