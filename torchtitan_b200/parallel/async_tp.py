"""Asynchronous tensor parallelism: the sequence all-gather before a
column-parallel GEMM and the reduce-scatter after a row-parallel GEMM are
decomposed into a ring of point-to-point transfers, each overlapped with the
GEMM of the chunk already present (the collective-matmul decomposition the
reference gets from Inductor's micro-pipeline pass,
``distributed/tensor_parallel.py:191-204``; here it is explicit, no compiler).

* ``AG -> GEMM`` (column-parallel, sequence-parallel input): each rank starts
  with its own sequence shard, multiplies it, and meanwhile passes the shard
  it holds to the left neighbour / receives the next one from the right; after
  ``tp - 1`` hops every shard has been multiplied once and the full gathered
  input has been assembled for the weight gradient.
* ``GEMM -> RS`` (row-parallel): rank ``r`` computes, at step ``i``, the
  partial product of output chunk ``(r + i + 1) % tp``, adds the partial sum
  received from the right neighbour and forwards it to the left one; at the
  last step it keeps its own fully reduced chunk ``r``.  The GEMM of step
  ``i + 1`` overlaps the transfer of step ``i``.

Backward of one is the other: d(AG->GEMM)/dx is a GEMM->RS of the output
gradient and d(GEMM->RS)/dx an AG->GEMM.  Transfers are ``batch_isend_irecv``
(NCCL on GPU, gloo on CPU), whose waits order the compute stream after each
hop.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from torchtitan_b200 import ops

ENABLED = False


def _exchange(send: torch.Tensor, group, rank: int, ws: int) -> tuple[torch.Tensor, list]:
    """Send ``send`` to the left neighbour, receive the same shape from the right one (async)."""
    recv = torch.empty_like(send)
    left = dist.get_global_rank(group, (rank - 1) % ws)
    right = dist.get_global_rank(group, (rank + 1) % ws)
    ops_ = [dist.P2POp(dist.isend, send, left, group), dist.P2POp(dist.irecv, recv, right, group)]
    return recv, dist.batch_isend_irecv(ops_)


def ring_ag_matmul(x: torch.Tensor, w: torch.Tensor, group) -> tuple[torch.Tensor, torch.Tensor]:
    """``all_gather_seq(x) @ w.T`` overlapped; returns (output [B,S,N], gathered input [B,S,K])."""
    ws, r = dist.get_world_size(group), dist.get_rank(group)
    s = x.shape[1]
    outs: list[torch.Tensor | None] = [None] * ws
    gathered: list[torch.Tensor | None] = [None] * ws
    cur = x.contiguous()
    for i in range(ws):
        src = (r + i) % ws  # the shard held at step i came from rank r + i
        reqs = []
        if i < ws - 1:
            nxt, reqs = _exchange(cur, group, r, ws)
        outs[src] = ops.linear(cur, w)
        gathered[src] = cur
        for q in reqs:
            q.wait()
        if i < ws - 1:
            cur = nxt
    assert all(o is not None for o in outs) and s * ws == sum(g.shape[1] for g in gathered)
    return torch.cat(outs, 1), torch.cat(gathered, 1)


def ring_matmul_rs(x: torch.Tensor, w: torch.Tensor, group) -> torch.Tensor:
    """``reduce_scatter_seq(x @ w.T)`` overlapped; x is [B, S, K], returns [B, S/tp, N]."""
    ws, r = dist.get_world_size(group), dist.get_rank(group)
    S = x.shape[1]
    s = S // ws
    acc = None
    for i in range(ws):
        c = (r + i + 1) % ws
        part = ops.linear(x[:, c * s:(c + 1) * s].contiguous(), w)
        if acc is not None:
            for q in reqs:
                q.wait()
            part = part + acc
        if i == ws - 1:
            return part
        acc, reqs = _exchange(part.contiguous(), group, r, ws)
    raise AssertionError("unreachable")


class AGMatmul(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, group):
        y, x_full = ring_ag_matmul(x, w, group)
        ctx.save_for_backward(x_full, w)
        ctx.group = group
        return y

    @staticmethod
    def backward(ctx, dy):
        x_full, w = ctx.saved_tensors
        dy = dy.contiguous()
        dx = ring_matmul_rs(dy, w.t().contiguous(), ctx.group)
        dw = ops.matmul(dy.reshape(-1, dy.shape[-1]).t().contiguous(), x_full.reshape(-1, x_full.shape[-1]))
        return dx, dw.to(w.dtype), None


class MatmulRS(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, group):
        ctx.save_for_backward(x, w)
        ctx.group = group
        return ring_matmul_rs(x.contiguous(), w, group)

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        dx, dy_full = ring_ag_matmul(dy.contiguous(), w.t().contiguous(), ctx.group)
        dw = ops.matmul(dy_full.reshape(-1, dy_full.shape[-1]).t().contiguous(), x.reshape(-1, x.shape[-1]))
        return dx, dw.to(w.dtype), None


def ag_matmul(x, w, group):
    """On B200s over NCCL the fused kernel (``parallel/tp_fused.py``); else the P2P ring."""
    from . import tp_fused

    if tp_fused.fused_available(x, group) and tp_fused.shapes_ok(x, w.shape[0], w.shape[1]):
        return tp_fused.FusedAGMatmul.apply(x, w, group)
    return AGMatmul.apply(x, w, group)


def matmul_rs(x, w, group):
    from . import tp_fused

    if tp_fused.fused_available(x, group) and tp_fused.shapes_ok(x, w.shape[0], w.shape[1]):
        return tp_fused.FusedMatmulRS.apply(x, w, group)
    return MatmulRS.apply(x, w, group)
