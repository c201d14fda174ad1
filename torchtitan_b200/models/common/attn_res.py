"""Block Attention Residuals (parity: reference
``experiments/attention_residual/attn_res.py:48-116``).

Instead of ``h = h + f(h)``, a layer's input is a learned softmax mixture of
the *block outputs* so far: the residual stream is cut into blocks of layers;
``V`` stacks the completed block sums and the current partial sum, keys are
``RMSNorm(V)``, and a per-layer pseudo-query ``w`` (zero-initialised, so the
mixture starts uniform) scores them:

    h = sum_n softmax_n(<w, RMSNorm(V_n)>) V_n

With one block per layer it is Full AttnRes.
"""
from __future__ import annotations

import torch

from .layers import RMSNorm, _local


def block_attn_res(blocks: list[torch.Tensor], partial: torch.Tensor, query: torch.Tensor, norm: RMSNorm):
    """softmax_n(<w, RMSNorm(V_n)>) weighted sum of V = blocks + [partial] (all [B,T,D])."""
    V = torch.stack(blocks + [partial], 0)
    Kn = norm(V)
    w = _local(query).reshape(-1).to(Kn.dtype)
    logits = torch.einsum("d,nbtd->nbt", w, Kn).float()
    return torch.einsum("nbt,nbtd->btd", torch.softmax(logits, 0).to(V.dtype), V)


def pack_state(state) -> torch.Tensor:
    """(completed blocks, partial block) -> one ``[n_blocks + 1, B, S, D]`` tensor, the form a
    pipeline stage sends to the next one (its shape is fixed per stage boundary)."""
    blocks, partial = state
    return torch.stack(list(blocks) + [partial])


def unpack_state(x: torch.Tensor):
    """Inverse of ``pack_state``; a plain ``[B, S, D]`` hidden state starts with no blocks."""
    if x.dim() == 3:
        return [], x
    parts = list(x.unbind(0))
    return parts[:-1], parts[-1]
