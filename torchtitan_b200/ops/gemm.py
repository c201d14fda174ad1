"""Dense GEMM on tcgen05 (``csrc/gemm_tcgen05.cu``) with autograd.

``ext().gemm(A, B, a_mn_major, b_mn_major)`` computes ``D[M,N] = sum_k A(m,k) B(n,k)``
in bf16 with fp32 accumulation in TMEM.  A is given either as ``[M,K]``
(K-major) or ``[K,M]`` (M-major); B as ``[N,K]`` or ``[K,N]``.  All three
GEMMs of a linear layer map onto it without transposes:

  forward  y  = x  @ w.T : A = x  [M,K] K-major,  B = w [N,K] K-major
  dgrad    dx = dy @ w   : A = dy [M,N] K-major,  B = w [N,K] read N-major
  wgrad    dw = dy.T @ x : A = dy [M,N] M-major,  B = x [M,K] read N-major

The forward GEMM is a registered custom op (``torch.ops.tt_b200.gemm``) so
selective activation checkpointing can decide per call whether to keep its
output.
"""
from __future__ import annotations

import torch

from . import _ext


@torch.library.custom_op("tt_b200::gemm", mutates_args=())
def gemm(a: torch.Tensor, b: torch.Tensor, a_mn_major: bool, b_mn_major: bool) -> torch.Tensor:
    return _ext.ext().gemm(a, b, a_mn_major, b_mn_major)


@gemm.register_fake
def _(a, b, a_mn_major, b_mn_major):
    m = a.shape[1] if a_mn_major else a.shape[0]
    n = b.shape[1] if b_mn_major else b.shape[0]
    return a.new_empty((m, n))


def _plain(t: torch.Tensor) -> torch.Tensor:
    return t.to_local() if type(t).__name__ == "DTensor" else t


class _Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w):
        x2 = x.reshape(-1, x.shape[-1])
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        wc = w if w.is_contiguous() else w.contiguous()
        y = torch.ops.tt_b200.gemm(x2, wc, False, False)
        ctx.save_for_backward(x2, wc)
        ctx.wdtype = w.dtype
        return y.view(*x.shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x2, w = ctx.saved_tensors
        dy2 = dy.reshape(-1, dy.shape[-1])
        if not dy2.is_contiguous():
            dy2 = dy2.contiguous()
        dx = dw = None
        if ctx.needs_input_grad[0]:
            dx = _ext.ext().gemm(dy2, w, False, True).view(*dy.shape[:-1], w.shape[1])
        if ctx.needs_input_grad[1]:
            dw = _ext.ext().gemm(dy2, x2, True, True)
        return dx, dw


def linear(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """``x @ w.T`` (no bias).  CPU tensors use ``F.linear``."""
    if not x.is_cuda:
        return torch.nn.functional.linear(x, w)
    if x.dtype != w.dtype:
        x = x.to(w.dtype)
    n, k = w.shape
    pn, pk = (-n) % 8, (-k) % 8
    if pn or pk:
        # TMA rows must be 16-byte multiples: zero-pad the feature dims (exact) and slice
        F = torch.nn.functional
        y = _Linear.apply(F.pad(x, (0, pk)) if pk else x, F.pad(w, (0, pk, 0, pn)))
        return y[..., :n] if pn else y
    return _Linear.apply(x, w)


class _Matmul(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a, b):
        ctx.save_for_backward(a, b)
        return _ext.ext().gemm(a.contiguous(), b.contiguous(), False, True)

    @staticmethod
    def backward(ctx, d):
        a, b = ctx.saved_tensors
        d = d.contiguous()
        da = _ext.ext().gemm(d, b.contiguous(), False, False) if ctx.needs_input_grad[0] else None
        db = _ext.ext().gemm(a.contiguous(), d, True, True) if ctx.needs_input_grad[1] else None
        return da, db


def bmm_grouped(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Batched ``a @ b`` for equal-shape stacks a [E, m, k], b [E, k, n] (no autograd) as ONE
    grouped tcgen05 GEMM: the grouped-reduction mode computes D_g = A_g^T B_g over row ranges
    of stacked operands, so A_g = a_g^T and B_g = b_g."""
    E, m, k = a.shape
    n = b.shape[-1]
    at = a.mT.contiguous().reshape(E * k, m)
    bt = b.contiguous().reshape(E * k, n)
    ks = torch.arange(0, E * k, k, dtype=torch.int32, device=a.device)
    kl = torch.full((E,), k, dtype=torch.int32, device=a.device)
    return _ext.ext().gemm_grouped_k(at, bt, ks, kl)


def matmul(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """2-D ``a @ b`` (bf16 on CUDA); 3-D stacks go through one grouped GEMM when no gradient
    is needed and the shapes allow it (row lengths multiples of 8), else a loop."""
    if not a.is_cuda:
        return a @ b
    if a.dim() > 2:
        if (a.dim() == 3 and b.dim() == 3 and a.shape[0] == b.shape[0] and not torch.is_grad_enabled()
                and a.shape[1] % 8 == 0 and b.shape[2] % 8 == 0):
            return bmm_grouped(a.bfloat16(), b.bfloat16()).to(a.dtype)
        return torch.stack([matmul(x, y) for x, y in zip(a.unbind(0), b.unbind(0))])
    if a.dtype != torch.bfloat16:
        return _Matmul.apply(a.bfloat16(), b.bfloat16()).to(a.dtype)
    return _Matmul.apply(a, b)
