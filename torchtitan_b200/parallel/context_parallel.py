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


# ------------------------------------------- Ulysses on the fused AG->GEMM / GEMM->RS kernels
# Ulysses shards attention by heads over the cp group with the full sequence per rank. The
# same sharding follows from sequence-parallel head-parallel projections: rank r computes
#   q_r, k_r, v_r = AllGather_seq(x) . W{q,k,v}[heads_r]^T      [B, S, H/cp, D]
#   out_r         = ReduceScatter_seq(o_r . Wo[:, heads_r]^T)     [B, S/cp, dim]
# with each collective inside one persistent tcgen05 GEMM over NVLink peer memory
# (``parallel/tp_fused.py``). The weights stay replicated over cp: rank r's gradient covers its
# head slice over the whole sequence (zero elsewhere) and the FSDP reduction over
# dp_shard x cp sums the slices, which equals the a2a formulation's per-sequence-shard sum.
# Per rank the GEMM FLOPs are those of the a2a form; the bytes over NVLink are the gathered
# input and the reduce-scattered output instead of the q/k/v and o shards.
_ROPE_FULL: dict = {}


def _gather_seq_table(t: torch.Tensor, group) -> torch.Tensor:
    """cos / sin of the local positions -> the full sequence (rank order = sequence order)."""
    key = (t.data_ptr(), tuple(t.shape), group.group_name)
    hit = _ROPE_FULL.get(key)
    if hit is not None and hit[0] is t:
        return hit[1]
    cp = dist.get_world_size(group)
    parts = [torch.empty_like(t) for _ in range(cp)]
    dist.all_gather(parts, t.contiguous(), group=group)
    full = torch.cat(parts, dim=t.dim() - 2)
    _ROPE_FULL.clear()  # one table pair per step is live
    _ROPE_FULL[key] = (t, full)
    return full


def _ulysses_fused_ok(attn, x, group) -> bool:
    from torchtitan_b200.parallel import tp_fused

    if not tp_fused.fused_available(x, group) or x.dtype != torch.bfloat16:
        return False
    cp = dist.get_world_size(group)
    hq, hk = attn.n_heads, attn.n_kv_heads
    if hq % cp or hk % cp or getattr(attn, "q_norm", None) is not None:
        return False
    lins = (attn.wq, attn.wk, attn.wv, attn.wo)
    if any(getattr(l, "bias", None) is not None or getattr(l, "tp_mode", None) for l in lins):
        return False
    D = attn.head_dim
    return (tp_fused.shapes_ok(x, hq // cp * D, x.shape[-1]) and tp_fused.shapes_ok(x, hk // cp * D, x.shape[-1])
            and (hq // cp * D) % 64 == 0)


def ulysses_fused_forward(attn, x, cos, sin, group):
    """Attention of ``attn`` (wq/wk/wv/wo, RoPE, causal) on sequence-sharded ``x``
    [B, S/cp, dim] with the Ulysses head sharding carried by the fused kernels."""
    from torchtitan_b200.models.common.layers import _local
    from torchtitan_b200.parallel.tp_fused import FusedAGMatmul, FusedMatmulRS

    cp, r = dist.get_world_size(group), dist.get_rank(group)
    D = attn.head_dim
    hq, hk = attn.n_heads // cp, attn.n_kv_heads // cp
    wq, wk, wv, wo = (_local(l.weight).to(x.dtype) for l in (attn.wq, attn.wk, attn.wv, attn.wo))
    B = x.shape[0]
    q = FusedAGMatmul.apply(x, wq[r * hq * D:(r + 1) * hq * D], group).view(B, -1, hq, D)
    k = FusedAGMatmul.apply(x, wk[r * hk * D:(r + 1) * hk * D], group).view(B, -1, hk, D)
    v = FusedAGMatmul.apply(x, wv[r * hk * D:(r + 1) * hk * D], group).view(B, -1, hk, D)
    cf, sf = _gather_seq_table(cos, group), _gather_seq_table(sin, group)
    q, k = ops.rope(q, cf, sf), ops.rope(k, cf, sf)
    o = attn.inner_attention(q, k, v, None)
    return FusedMatmulRS.apply(o.reshape(B, o.shape[1], hq * D), wo[:, r * hq * D:(r + 1) * hq * D].contiguous(),
                               group)


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
        if method == "ulysses":
            m.cp_group = group  # enables the fused-kernel path where it applies (see Attention.forward)


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
