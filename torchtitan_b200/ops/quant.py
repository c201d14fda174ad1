"""Low-precision number formats used by the Float8 / MXFP8 training recipes.

* MXFP8 (OCP Microscaling v1.0): blocks of 32 consecutive elements along the
  contraction dimension share one power-of-two scale stored as E8M0; elements
  are FP8 E4M3.  The scale exponent uses round-to-ceiling of
  ``log2(amax / 448)`` ("RCEIL"), so no element overflows E4M3 after scaling.
* Float8 tensorwise / rowwise: one fp32 scale ``448 / amax`` per tensor or per
  row, E4M3 elements.

Functions return the *dequantized* tensor (what the GEMM effectively
multiplies) together with the raw codes, so a block-scaled GEMM and the
emulation path see bit-identical operands.
"""
from __future__ import annotations

import torch

E4M3_MAX = 448.0
MX_BLOCK = 32


def mx_quantize(x: torch.Tensor, block: int = MX_BLOCK) -> tuple[torch.Tensor, torch.Tensor]:
    """Quantize along the last dim in blocks of ``block``: returns (fp8 e4m3 codes, e8m0 exponents uint8)."""
    if x.shape[-1] % block:
        raise ValueError(f"MX quantization needs the last dim divisible by {block}, got {x.shape[-1]}")
    xb = x.float().reshape(*x.shape[:-1], x.shape[-1] // block, block)
    amax = xb.abs().amax(-1, keepdim=True)
    # RCEIL: smallest power of two s with amax / s <= 448, i.e. ceil(log2(amax / 448)), taken
    # exactly from the binary exponent (frexp: y = m * 2^p, m in [0.5, 1)); zero blocks get 2^-127
    m, p = torch.frexp(amax / E4M3_MAX)
    exp = torch.where(m == 0.5, p - 1, p).float().clamp(-127, 127)
    exp = torch.where(amax == 0, torch.full_like(exp, -127.0), exp)
    scaled = (xb * torch.exp2(-exp)).clamp(-E4M3_MAX, E4M3_MAX)
    codes = scaled.to(torch.float8_e4m3fn).reshape(x.shape)
    return codes, (exp.squeeze(-1) + 127).to(torch.uint8)


def mx_dequantize(codes: torch.Tensor, scales: torch.Tensor, dtype=torch.bfloat16, block: int = MX_BLOCK):
    x = codes.float().reshape(*codes.shape[:-1], codes.shape[-1] // block, block)
    x = x * torch.exp2(scales.float() - 127)[..., None]
    return x.reshape(codes.shape).to(dtype)


def mx_fake_quant(x: torch.Tensor, dim: int = -1, dtype=None) -> torch.Tensor:
    """Quantize-dequantize with blocks along ``dim``."""
    t = x.transpose(dim, -1) if dim not in (-1, x.dim() - 1) else x
    q, s = mx_quantize(t)
    out = mx_dequantize(q, s, dtype or x.dtype)
    return out.transpose(dim, -1) if dim not in (-1, x.dim() - 1) else out


def float8_fake_quant(x: torch.Tensor, granularity: str = "tensorwise", dim: int = -1) -> torch.Tensor:
    """E4M3 quantize-dequantize with one scale per tensor or per row (rows = slices along ``dim``)."""
    xf = x.float()
    if granularity == "tensorwise":
        amax = xf.abs().amax()
    else:
        amax = xf.abs().amax(dim=dim, keepdim=True)
    scale = E4M3_MAX / amax.clamp_min(1e-12)
    q = (xf * scale).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn)
    return (q.float() / scale).to(x.dtype)
