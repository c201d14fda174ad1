"""Context parallelism: Ulysses (sequence<->head all-to-all) and ring attention.

* **Ulysses** (not in the reference; needed for long-context Kimi-Linear):
  q/k/v arrive sequence-sharded ``[B, S/cp, H, D]``; one all-to-all turns
  them into head-sharded full sequences ``[B, S, H/cp, D]``, attention (or
  any full-sequence mixer, e.g. KDA) runs locally, and the inverse
  all-to-all restores sequence shards.  Requires ``cp | H`` (and ``cp | Hkv``).
* **Ring / all-gather** (parity with the reference's ``_ContextParallel``
  allgather rotation, ``torchtitan/distributed/context_parallel.py:51-259``):
  K/V are all-gathered along the sequence; each rank's queries are two
  head-tail chunks (load balancing for the causal mask) that attend to the
  K/V prefix ending at their own position.

Input sharding for both is produced by ``prepare_context_parallel_input``.
"""
from __future__ import annotations

from typing import Any

import torch
import torch.distributed as dist

from torchtitan_b200 import ops


# ----------------------------------------------------------------- all-to-all
def _a2a_seq_to_head(x: torch.Tensor, group) -> torch.Tensor:
    """[B, S/cp, H, D] -> [B, S, H/cp, D]."""
    cp = dist.get_world_size(group)
    B, s, H, D = x.shape
    send = x.reshape(B, s, cp, H // cp, D).permute(2, 0, 1, 3, 4).contiguous()  # [cp, B, s, H/cp, D]
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    return recv.permute(1, 0, 2, 3, 4).reshape(B, cp * s, H // cp, D)


def _a2a_head_to_seq(x: torch.Tensor, group) -> torch.Tensor:
    """[B, S, H/cp, D] -> [B, S/cp, H, D]."""
    cp = dist.get_world_size(group)
    B, S, h, D = x.shape
    send = x.reshape(B, cp, S // cp, h, D).permute(1, 0, 2, 3, 4).contiguous()  # [cp, B, s, h, D]
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    return recv.permute(1, 2, 0, 3, 4).reshape(B, S // cp, cp * h, D)


class _SeqToHead(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return _a2a_seq_to_head(x, group)

    @staticmethod
    def backward(ctx, g):
        return _a2a_head_to_seq(g.contiguous(), ctx.group), None


class _HeadToSeq(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return _a2a_head_to_seq(x, group)

    @staticmethod
    def backward(ctx, g):
        return _a2a_seq_to_head(g.contiguous(), ctx.group), None


def seq_to_head(x, group):
    return _SeqToHead.apply(x, group)


def head_to_seq(x, group):
    return _HeadToSeq.apply(x, group)


def ulysses_hook(group):
    def hook(inner, q, k, v, masks):
        q, k, v = (seq_to_head(t, group) for t in (q, k, v))
        o = inner(q, k, v, masks)
        return head_to_seq(o, group)

    return hook


# ------------------------------------------------------------ ring (allgather)
class _AllGatherSeqCP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        ws = dist.get_world_size(group)
        xs = x.transpose(0, 1).contiguous()
        out = torch.empty((ws * xs.shape[0],) + tuple(xs.shape[1:]), dtype=x.dtype, device=x.device)
        dist.all_gather_into_tensor(out, xs, group=group)
        return out.transpose(0, 1)

    @staticmethod
    def backward(ctx, g):
        ws = dist.get_world_size(ctx.group)
        gs = g.transpose(0, 1).contiguous()
        out = torch.empty((gs.shape[0] // ws,) + tuple(gs.shape[1:]), dtype=g.dtype, device=g.device)
        dist.reduce_scatter_tensor(out, gs, group=ctx.group)
        return out.transpose(0, 1), None


def headtail_order(cp: int) -> list[int]:
    """Chunk order in the gathered sequence: rank r holds chunks r and 2cp-1-r."""
    order = []
    for r in range(cp):
        order += [r, 2 * cp - 1 - r]
    return order


def ring_hook(group, load_balance: bool = True):
    cp = dist.get_world_size(group)
    rank = dist.get_rank(group)

    def hook(inner, q, k, v, masks):
        kf = _AllGatherSeqCP.apply(k, group)  # [B, cp*s, Hk, D] in head-tail order
        vf = _AllGatherSeqCP.apply(v, group)
        if load_balance:
            order = headtail_order(cp)
            c = q.shape[1] // 2
            inv = [order.index(j) for j in range(2 * cp)]
            kf = torch.cat([kf[:, inv[j] * c:(inv[j] + 1) * c] for j in range(2 * cp)], 1)
            vf = torch.cat([vf[:, inv[j] * c:(inv[j] + 1) * c] for j in range(2 * cp)], 1)
            outs = []
            for half, chunk in enumerate((rank, 2 * cp - 1 - rank)):
                qc = q[:, half * c:(half + 1) * c]
                end = (chunk + 1) * c
                outs.append(ops.attention(qc, kf[:, :end], vf[:, :end], causal=True))
            return torch.cat(outs, 1)
        s = q.shape[1]
        end = (rank + 1) * s
        return ops.attention(q, kf[:, :end], vf[:, :end], causal=True)

    return hook


def apply_cp_to_attention_modules(modules: list, cp_mesh, method: str = "ring", load_balance: bool = True) -> None:
    group = cp_mesh.get_group()
    for m in modules:
        m.cp_hook = ulysses_hook(group) if method == "ulysses" else ring_hook(group, load_balance)


def prepare_context_parallel_input(inputs: torch.Tensor, labels: torch.Tensor, extra_kwargs: dict[str, Any],
                                   cp_mesh, device, load_balancer: str | None = "headtail",
                                   method: str = "ring") -> tuple[torch.Tensor, torch.Tensor, dict[str, Any]]:
    """Shard tokens/labels/positions along the sequence for this CP rank."""
    cp, rank = cp_mesh.size(), cp_mesh.get_local_rank()
    S = inputs.shape[1]
    pos = extra_kwargs.get("positions")
    if pos is None:
        pos = torch.arange(S, device=inputs.device).expand(inputs.shape[0], S)
    if method == "ring" and load_balancer == "headtail":
        c = S // (2 * cp)
        sl = [slice(rank * c, (rank + 1) * c), slice((2 * cp - 1 - rank) * c, (2 * cp - rank) * c)]
        pick = lambda t: torch.cat([t[:, s] for s in sl], 1)  # noqa: E731
    else:
        s = S // cp
        pick = lambda t: t[:, rank * s:(rank + 1) * s]  # noqa: E731
    extra_kwargs = dict(extra_kwargs)
    extra_kwargs["positions"] = pick(pos)
    return pick(inputs), pick(labels), extra_kwargs
