"""Causal GQA flash attention (``csrc/flash_attn.cu``) with autograd.

Layout is ``[B, S, H, D]`` (sequence-major, as produced by the QKV GEMM), so
no transposes are needed around the kernel.  Forward returns the output and
the per-row log-sum-exp (fp32, ``[B, H, S]`` padded to a multiple of 64), which backward uses to
recompute probabilities tile by tile.  ``Dq`` may differ from ``Dv`` (MLA:
192 / 128).  The forward is a registered custom op so selective activation
checkpointing can keep its output.
"""
from __future__ import annotations

import math

import torch

from . import _ext
from . import reference as _ref


@torch.library.custom_op("tt_b200::attn_fwd", mutates_args=())
def attn_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool, scale: float,
             doc_start: torch.Tensor | None = None,
             doc_end: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    o, lse = _ext.ext().attn_fwd(q, k, v, causal, scale, doc_start, doc_end)
    return o, lse


@attn_fwd.register_fake
def _(q, k, v, causal, scale, doc_start=None, doc_end=None):
    B, S, H, _ = q.shape
    return q.new_empty((B, S, H, v.shape[-1])), q.new_empty((B, H, (S + 63) // 64 * 64), dtype=torch.float32)


class _Attn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, causal, scale, doc_start=None, doc_end=None):
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        o, lse = torch.ops.tt_b200.attn_fwd(q, k, v, causal, scale, doc_start, doc_end)
        ctx.save_for_backward(q, k, v, o, lse, doc_start, doc_end)
        ctx.causal, ctx.scale = causal, scale
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse, doc_start, doc_end = ctx.saved_tensors
        dq, dk, dv = _ext.ext().attn_bwd(do.contiguous(), q, k, v, o, lse, ctx.causal, ctx.scale,
                                         doc_start=doc_start, doc_end=doc_end)
        return dq, dk, dv, None, None, None, None


_SUPPORTED = ((64, 64), (128, 128), (192, 128))


def _padded_dims(dqk: int, dv: int) -> tuple[int, int]:
    for a, b in _SUPPORTED:
        if dqk <= a and dv <= b:
            return a, b
    raise ValueError(f"attention head dims ({dqk}, {dv}) exceed the supported maximum (192, 128)")


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = True,
              scale: float | None = None) -> torch.Tensor:
    scale = float(scale if scale is not None else 1.0 / math.sqrt(q.shape[-1]))
    if not q.is_cuda:
        return _ref.attention(q, k, v, causal, scale)
    dqk, dv = q.shape[-1], v.shape[-1]
    pq, pv = _padded_dims(dqk, dv)
    if (pq, pv) != (dqk, dv):
        # zero-padding q/k leaves every dot product unchanged; extra v columns are dropped
        F = torch.nn.functional
        q, k = F.pad(q, (0, pq - dqk)), F.pad(k, (0, pq - dqk))
        v = F.pad(v, (0, pv - dv))
        return _Attn.apply(q, k, v, causal, scale)[..., :dv]
    return _Attn.apply(q, k, v, causal, scale)


class _AttnLse(torch.autograd.Function):
    """Attention that also returns the per-row log-sum-exp ``[B, S, H]`` (natural log) and
    backpropagates through both outputs: a gradient on the LSE shifts delta by -dlse."""

    @staticmethod
    def forward(ctx, q, k, v, causal, scale):
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        o, lse = torch.ops.tt_b200.attn_fwd(q, k, v, causal, scale)
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.causal, ctx.scale = causal, scale
        S = q.shape[1]
        return o, lse[:, :, :S].transpose(1, 2)

    @staticmethod
    def backward(ctx, do, dlse):
        q, k, v, o, lse = ctx.saved_tensors
        full = None
        if dlse is not None:
            full = torch.zeros_like(lse)
            full[:, :, : q.shape[1]] = dlse.transpose(1, 2).float()
        dq, dk, dv = _ext.ext().attn_bwd(do.contiguous(), q, k, v, o, lse, ctx.causal, ctx.scale, full)
        return dq, dk, dv, None, None


def _attention_lse_ref(q, k, v, causal, scale):
    H, Hk = q.shape[2], k.shape[2]
    if Hk != H:
        k, v = k.repeat_interleave(H // Hk, dim=2), v.repeat_interleave(H // Hk, dim=2)
    s = torch.einsum("bshd,bthd->bhst", q.float(), k.float()) * scale
    if causal:
        Sq, Sk = q.shape[1], k.shape[1]
        keep = torch.ones(Sq, Sk, dtype=torch.bool, device=q.device).tril(diagonal=Sk - Sq)
        s = s.masked_fill(~keep, float("-inf"))
    lse = torch.logsumexp(s, -1)
    o = torch.einsum("bhst,bthd->bshd", torch.exp(s - lse[..., None]), v.float())
    return o.to(q.dtype), lse.transpose(1, 2)


def attention_with_lse(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = True,
                       scale: float | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """(o [B,S,H,Dv], lse [B,S,H] fp32); both differentiable."""
    scale = float(scale if scale is not None else 1.0 / math.sqrt(q.shape[-1]))
    if not q.is_cuda:
        return _attention_lse_ref(q, k, v, causal, scale)
    dqk, dv = q.shape[-1], v.shape[-1]
    pq, pv = _padded_dims(dqk, dv)
    if (pq, pv) != (dqk, dv):
        F = torch.nn.functional
        q, k = F.pad(q, (0, pq - dqk)), F.pad(k, (0, pq - dqk))
        v = F.pad(v, (0, pv - dv))
        o, lse = _AttnLse.apply(q, k, v, causal, scale)
        return o[..., :dv], lse
    return _AttnLse.apply(q, k, v, causal, scale)


def document_segments(doc_ids: torch.Tensor) -> list[list[tuple[int, int]]]:
    """[B, S] non-decreasing document ids -> per row, the (start, end) of each document."""
    B, S = doc_ids.shape
    change = torch.ones(B, S, dtype=torch.bool, device=doc_ids.device)
    change[:, 1:] = doc_ids[:, 1:] != doc_ids[:, :-1]
    rows = []
    for starts in change.cpu():
        s = starts.nonzero().flatten().tolist() + [S]
        rows.append(list(zip(s[:-1], s[1:])))
    return rows


def document_tables(doc_ids: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """[B, S] document ids (contiguous runs) -> (start, end) int32 [B, S] on the same device:
    the first position of each token's document and one past its last. Computed with scans on
    the device (no host synchronisation)."""
    B, S = doc_ids.shape
    idx = torch.arange(S, device=doc_ids.device, dtype=torch.int64).expand(B, S)
    first = torch.ones(B, S, dtype=torch.bool, device=doc_ids.device)
    first[:, 1:] = doc_ids[:, 1:] != doc_ids[:, :-1]
    start = torch.where(first, idx, torch.zeros_like(idx)).cummax(dim=1).values
    nxt = torch.where(first, idx, torch.full_like(idx, S))
    nxt = torch.cat([nxt[:, 1:], torch.full_like(nxt[:, :1], S)], dim=1)
    end = nxt.flip(1).cummin(dim=1).values.flip(1)
    return start.to(torch.int32).contiguous(), end.to(torch.int32).contiguous()


def document_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, doc_ids: torch.Tensor,
                       scale: float | None = None) -> torch.Tensor:
    """Causal attention within packed documents (reference ``models/common/attention.py:220``
    varlen path): q [B,S,H,D], k/v [B,S,Hk,D]; ``doc_ids`` [B,S] labels each token's
    document (contiguous runs).  On a GPU with head dims up to 128 this is one launch of the
    flash kernels with the block-causal mask applied inside them (per-token document start
    and end tables; query tiles skip key tiles of earlier documents, key tiles skip queries
    of later ones); otherwise each document runs on its own rows."""
    scale_v = float(scale if scale is not None else 1.0 / math.sqrt(q.shape[-1]))
    dqk, dv = q.shape[-1], v.shape[-1]
    if q.is_cuda and dqk <= 128 and dv <= 128 and q.shape[1] == k.shape[1]:
        start, end = document_tables(doc_ids)
        pq, pv = _padded_dims(dqk, dv)
        if (pq, pv) != (dqk, dv):
            F = torch.nn.functional
            qq, kk, vv = F.pad(q, (0, pq - dqk)), F.pad(k, (0, pq - dqk)), F.pad(v, (0, pv - dv))
            return _Attn.apply(qq, kk, vv, True, scale_v, start, end)[..., :dv]
        return _Attn.apply(q, k, v, True, scale_v, start, end)
    parts = []
    for b, segs in enumerate(document_segments(doc_ids)):
        for s0, s1 in segs:
            parts.append(attention(q[b:b + 1, s0:s1], k[b:b + 1, s0:s1], v[b:b + 1, s0:s1], True, scale))
    return torch.cat([p[0] for p in parts]).view(*q.shape[:-1], v.shape[-1])
