"""Grouped SwiGLU experts on the grouped tcgen05 GEMM.

Rows arrive sorted by expert with ``counts[e]`` rows each.  They are copied (one row
gather kernel; padding rows written as zeros) into a padded buffer where expert e's rows start at a multiple of 128 (the
GEMM's M tile), so every 128-row tile belongs to exactly one expert and every
expert's K range (for the weight gradient) is 128-aligned.  The layout is
computed on the device from ``counts`` with a fixed upper bound on the padded
size (rows + 127 * E), so no device-to-host synchronisation is needed.

  forward:  h1 = X W1[e]^T, h3 = X W3[e]^T, a = silu(h1) h3, Y = a W2[e]^T   (grouped rows)
  backward: da = dY W2[e],  dh1, dh3 = swiglu'(da),  dX = dh1 W1[e] + dh3 W3[e]
            dW2[e] = dY_e^T a_e,  dW1[e] = dh1_e^T X_e,  dW3[e] = dh3_e^T X_e    (grouped K)
"""
from __future__ import annotations

import torch

from . import _ext

TILE = 128


def padded_layout(counts: torch.Tensor, n_rows: int):
    """Returns (dest [n_rows] padded row of each input row, tile_group [P/128] int32,
    kstart [E] int32, klen [E] int32, P)."""
    E = counts.numel()
    counts = counts.to(torch.int64)
    padded = (counts + TILE - 1) // TILE * TILE
    pend = torch.cumsum(padded, 0)
    pstart = pend - padded
    start = torch.cumsum(counts, 0) - counts
    P = ((n_rows + (TILE - 1) * E) + TILE - 1) // TILE * TILE
    expert_of_row = torch.repeat_interleave(torch.arange(E, device=counts.device), counts, output_size=n_rows)
    dest = pstart[expert_of_row] + (torch.arange(n_rows, device=counts.device) - start[expert_of_row])
    tile_start = torch.arange(P // TILE, device=counts.device) * TILE
    g = torch.searchsorted(pend, tile_start, right=True)
    tile_group = torch.where(tile_start < pend[-1], g, torch.full_like(g, -1)).to(torch.int32)
    return dest, tile_group, pstart.to(torch.int32), padded.to(torch.int32), P


class _GroupedSwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w1, w2, w3, counts):
        ext = _ext.ext()
        E, H, D = w1.shape
        n = x.shape[0]
        dest, tg, kst, kln, P = padded_layout(counts, n)
        src_of = torch.full((P,), -1, dtype=torch.int64, device=x.device)  # padding rows read as zeros
        src_of[dest] = torch.arange(n, device=x.device)
        xp = ext.gather_rows(x, src_of)
        w1f, w3f, w2f = w1.reshape(E * H, D), w3.reshape(E * H, D), w2.reshape(E * D, H)
        h1 = ext.gemm_grouped_rows(xp, w1f, tg, H, H, False)
        h3 = ext.gemm_grouped_rows(xp, w3f, tg, H, H, False)
        a = ext.swiglu_fwd(h1, h3)
        yp = ext.gemm_grouped_rows(a, w2f, tg, D, D, False)
        ctx.save_for_backward(xp, h1, h3, a, w1, w2, w3, dest, src_of, tg, kst, kln)
        return ext.gather_rows(yp, dest)

    @staticmethod
    def backward(ctx, dy):
        ext = _ext.ext()
        xp, h1, h3, a, w1, w2, w3, dest, src_of, tg, kst, kln = ctx.saved_tensors
        E, H, D = w1.shape
        dyp = ext.gather_rows(dy.contiguous(), src_of)
        # dgrad through w2: B = W2[e] read as [D(red), H(out)] rows of the stacked [E*D, H]
        da = ext.gemm_grouped_rows(dyp, w2.reshape(E * D, H), tg, H, D, True)
        dh1, dh3 = ext.swiglu_bwd(da, h1, h3)
        dx = ext.gemm_grouped_rows(dh1, w1.reshape(E * H, D), tg, D, H, True)
        dx.add_(ext.gemm_grouped_rows(dh3, w3.reshape(E * H, D), tg, D, H, True))
        dw2 = ext.gemm_grouped_k(dyp, a, kst, kln)    # [E, D, H]
        dw1 = ext.gemm_grouped_k(dh1, xp, kst, kln)   # [E, H, D]
        dw3 = ext.gemm_grouped_k(dh3, xp, kst, kln)
        return ext.gather_rows(dx, dest), dw1.to(w1.dtype), dw2.to(w2.dtype), dw3.to(w3.dtype), None


class _MXGroupedSwiGLU(torch.autograd.Function):
    """Routed SwiGLU experts at MXFP8 rate: the forward GEMMs and both data-gradient GEMMs run
    on the block-scaled tcgen05 kernel in grouped-rows mode, every operand quantized (1x32
    E8M0 blocks) along its GEMM's contraction dim; the weight gradients stay in bf16 on the
    grouped-K kernel (high-precision weight gradient)."""

    @staticmethod
    def forward(ctx, x, w1, w2, w3, counts):
        from .mx_gemm import mx_gemm_grouped, mx_quantize

        ext = _ext.ext()
        E, H, D = w1.shape
        n = x.shape[0]
        dest, tg, kst, kln, P = padded_layout(counts, n)
        src_of = torch.full((P,), -1, dtype=torch.int64, device=x.device)
        src_of[dest] = torch.arange(n, device=x.device)
        xp = ext.gather_rows(x, src_of)
        qx = mx_quantize(xp)
        h1 = mx_gemm_grouped(*qx, *mx_quantize(w1.reshape(E * H, D)), tg, H)
        h3 = mx_gemm_grouped(*qx, *mx_quantize(w3.reshape(E * H, D)), tg, H)
        a = ext.swiglu_fwd(h1, h3)
        yp = mx_gemm_grouped(*mx_quantize(a), *mx_quantize(w2.reshape(E * D, H)), tg, D)
        ctx.save_for_backward(xp, h1, h3, a, w1, w2, w3, dest, src_of, tg, kst, kln)
        return ext.gather_rows(yp, dest)

    @staticmethod
    def backward(ctx, dy):
        from .mx_gemm import mx_gemm_grouped, mx_quantize

        ext = _ext.ext()
        xp, h1, h3, a, w1, w2, w3, dest, src_of, tg, kst, kln = ctx.saved_tensors
        E, H, D = w1.shape
        dyp = ext.gather_rows(dy.contiguous(), src_of)
        # da = dY W2[e]: contraction over D, so W2[e]^T [H, D] is quantized along D
        da = mx_gemm_grouped(*mx_quantize(dyp), *mx_quantize(w2.transpose(1, 2).reshape(E * H, D).contiguous()),
                             tg, H)
        dh1, dh3 = ext.swiglu_bwd(da, h1, h3)
        # dX = dh1 W1[e] + dh3 W3[e]: contraction over H, W^T [D, H] quantized along H
        dx = mx_gemm_grouped(*mx_quantize(dh1), *mx_quantize(w1.transpose(1, 2).reshape(E * D, H).contiguous()),
                             tg, D)
        dx.add_(mx_gemm_grouped(*mx_quantize(dh3),
                                *mx_quantize(w3.transpose(1, 2).reshape(E * D, H).contiguous()), tg, D))
        dw2 = ext.gemm_grouped_k(dyp, a, kst, kln)
        dw1 = ext.gemm_grouped_k(dh1, xp, kst, kln)
        dw3 = ext.gemm_grouped_k(dh3, xp, kst, kln)
        return ext.gather_rows(dx, dest), dw1.to(w1.dtype), dw2.to(w2.dtype), dw3.to(w3.dtype), None


def mx_grouped_swiglu_cuda(x, w1, w2, w3, counts):
    """MXFP8 routed experts on CUDA; expert dims (D, H) must be multiples of 128."""
    dt = torch.bfloat16
    return _MXGroupedSwiGLU.apply(x.to(dt).contiguous(), w1.to(dt).contiguous(), w2.to(dt).contiguous(),
                                  w3.to(dt).contiguous(), counts)


def grouped_swiglu_cuda(x, w1, w2, w3, counts):
    dt = torch.bfloat16
    return _GroupedSwiGLU.apply(x.to(dt).contiguous(), w1.to(dt).contiguous(), w2.to(dt).contiguous(),
                                w3.to(dt).contiguous(), counts)


def expert_segments(counts: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, int]:
    """Padded expert-major layout for ``counts`` rows per expert: (tile_group [P/128],
    kstart [E], klen [E], P) with every expert segment starting on a 128-row boundary."""
    counts = counts.to(torch.int64)
    padded = (counts + TILE - 1) // TILE * TILE
    pend = torch.cumsum(padded, 0)
    P = int(pend[-1]) if counts.numel() else 0
    tile_start = torch.arange(P // TILE, device=counts.device) * TILE
    tg = torch.searchsorted(pend, tile_start, right=True).to(torch.int32)
    return tg, (pend - padded).to(torch.int32), padded.to(torch.int32), P


class _GroupedSwiGLUPadded(torch.autograd.Function):
    """Grouped SwiGLU on rows already laid out in padded expert segments (padding rows
    zero), e.g. written there directly by a peer-memory expert-parallel dispatch."""

    @staticmethod
    def forward(ctx, xp, w1, w2, w3, tg, kst, kln):
        ext = _ext.ext()
        E, H, D = w1.shape
        h1 = ext.gemm_grouped_rows(xp, w1.reshape(E * H, D), tg, H, H, False)
        h3 = ext.gemm_grouped_rows(xp, w3.reshape(E * H, D), tg, H, H, False)
        a = ext.swiglu_fwd(h1, h3)
        yp = ext.gemm_grouped_rows(a, w2.reshape(E * D, H), tg, D, D, False)
        ctx.save_for_backward(xp, h1, h3, a, w1, w2, w3, tg, kst, kln)
        return yp

    @staticmethod
    def backward(ctx, dyp):
        ext = _ext.ext()
        xp, h1, h3, a, w1, w2, w3, tg, kst, kln = ctx.saved_tensors
        E, H, D = w1.shape
        dyp = dyp.contiguous()
        da = ext.gemm_grouped_rows(dyp, w2.reshape(E * D, H), tg, H, D, True)
        dh1, dh3 = ext.swiglu_bwd(da, h1, h3)
        dx = ext.gemm_grouped_rows(dh1, w1.reshape(E * H, D), tg, D, H, True)
        dx.add_(ext.gemm_grouped_rows(dh3, w3.reshape(E * H, D), tg, D, H, True))
        dw2 = ext.gemm_grouped_k(dyp, a, kst, kln)
        dw1 = ext.gemm_grouped_k(dh1, xp, kst, kln)
        dw3 = ext.gemm_grouped_k(dh3, xp, kst, kln)
        return dx, dw1.to(w1.dtype), dw2.to(w2.dtype), dw3.to(w3.dtype), None, None, None


def _grouped_swiglu_padded_ref(xp, w1, w2, w3, kst, kln):
    outs = []
    for e in range(w1.shape[0]):
        seg = xp[int(kst[e]):int(kst[e]) + int(kln[e])]
        h = torch.nn.functional.silu(seg @ w1[e].t()) * (seg @ w3[e].t())
        outs.append(h @ w2[e].t())
    return torch.cat(outs) if outs else xp.new_zeros(0, w2.shape[1])


def grouped_swiglu_padded(xp, w1, w2, w3, counts):
    """``xp``: [P, D] rows in the padded expert-major layout of ``counts`` (zero padding)."""
    tg, kst, kln, P = expert_segments(counts)
    if xp.shape[0] != P:
        raise ValueError(f"padded input has {xp.shape[0]} rows, layout needs {P}")
    if not xp.is_cuda:
        return _grouped_swiglu_padded_ref(xp, w1, w2, w3, kst, kln)
    dt = torch.bfloat16
    return _GroupedSwiGLUPadded.apply(xp.to(dt).contiguous(), w1.to(dt).contiguous(), w2.to(dt).contiguous(),
                                      w3.to(dt).contiguous(), tg, kst, kln)
