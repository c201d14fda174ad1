"""MXFP8 quantize + block-scaled GEMM (``csrc/mx_quant.cu``, ``csrc/gemm_mxfp8.cu``).

Storage: codes ``uint8 [R, Cp]`` (FP8 E4M3 bits, ``Cp`` = columns rounded up to
128, zero padded) and E8M0 scale bytes in the tcgen05 *blocked* layout: for row
block ``rb`` (128 rows) and column block ``cb`` (128 columns) a 512-byte record
at ``(rb * Cp/128 + cb) * 512`` holds the scale of row ``rb*128 + 32*m1 + m0``
and 32-column group ``4*cb + j`` at byte ``m0*16 + m1*4 + j``.  The CPU paths
below define the format (and serve as the reference in tests).
"""
from __future__ import annotations

import torch

from .quant import E4M3_MAX, mx_quantize as _mx_codes


def sf_byte_index(R: int, Cp: int) -> torch.Tensor:
    """[Rp, Cp/32] int64: byte offset of every (row, 32-column group) scale."""
    Rp = (R + 127) // 128 * 128
    r = torch.arange(Rp)[:, None]
    g = torch.arange(Cp // 32)[None, :]
    rin = r % 128
    return ((r // 128) * (Cp // 128) + g // 4) * 512 + (rin % 32) * 16 + (rin // 32) * 4 + g % 4


def mx_quantize_ref(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    R, C = x.shape
    Cp = (C + 127) // 128 * 128
    Rp = (R + 127) // 128 * 128
    xp = torch.zeros(R, Cp, dtype=torch.float32)
    xp[:, :C] = x.float().cpu()
    codes, e8 = _mx_codes(xp)                      # e8: [R, Cp/32] uint8
    e8[:, (C + 31) // 32:] = 127                   # groups wholly in the column padding: scale 2^0
    sf = torch.full((Rp * Cp // 32,), 127, dtype=torch.uint8)
    sf[sf_byte_index(R, Cp)[:R].reshape(-1)] = e8.reshape(-1)
    return codes.view(torch.uint8), sf


def mx_dequantize_ref(codes: torch.Tensor, sf: torch.Tensor) -> torch.Tensor:
    R, Cp = codes.shape
    e8 = sf.cpu()[sf_byte_index(R, Cp)[:R]]        # [R, Cp/32]
    vals = codes.cpu().view(torch.float8_e4m3fn).float().view(R, Cp // 32, 32)
    return (vals * torch.exp2(e8.float() - 127)[..., None]).view(R, Cp)


def mx_quantize(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    if x.is_cuda:
        from ._ext import ext

        return tuple(ext().mx_quantize(x.to(torch.bfloat16)))
    return mx_quantize_ref(x)


def mx_gemm(a: torch.Tensor, sfa: torch.Tensor, b: torch.Tensor, sfb: torch.Tensor) -> torch.Tensor:
    """A codes [M, Kp] x B codes [N, Kp] -> bf16 [M, N] with per-32 E8M0 scales on both."""
    if a.is_cuda:
        from ._ext import ext

        return ext().gemm_mxfp8(a, sfa, b, sfb)
    return (mx_dequantize_ref(a, sfa) @ mx_dequantize_ref(b, sfb).t()).to(torch.bfloat16)


def mx_gemm_grouped(a: torch.Tensor, sfa: torch.Tensor, b: torch.Tensor, sfb: torch.Tensor,
                    tile_group: torch.Tensor, n: int) -> torch.Tensor:
    """Grouped rows: A codes [P, Kp] (rows padded per group to 128) times group
    ``tile_group[i]`` of the stacked B codes [G*n, Kp] for every 128-row tile ``i``
    (negative: tile skipped, its rows undefined) -> bf16 [P, n]."""
    if a.is_cuda:
        from ._ext import ext

        return ext().gemm_mxfp8_grouped(a, sfa, b, sfb, tile_group, n)
    A, B = mx_dequantize_ref(a, sfa), mx_dequantize_ref(b, sfb)
    out = torch.zeros(a.shape[0], n)
    for i, g in enumerate(tile_group.tolist()):
        if g >= 0:
            out[i * 128:(i + 1) * 128] = A[i * 128:(i + 1) * 128] @ B[g * n:(g + 1) * n].t()
    return out.to(torch.bfloat16)


def mx_linear(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """``x @ w.T`` with both operands MXFP8-quantized along the contraction dim."""
    x2 = x.reshape(-1, x.shape[-1])
    qa, sa = mx_quantize(x2)
    qb, sb = mx_quantize(w)
    return mx_gemm(qa, sa, qb, sb).view(*x.shape[:-1], w.shape[0])


__all__ = ["E4M3_MAX", "mx_quantize", "mx_gemm", "mx_gemm_grouped", "mx_linear", "mx_quantize_ref", "mx_dequantize_ref",
           "sf_byte_index"]
