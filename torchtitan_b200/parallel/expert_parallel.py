"""Expert parallelism (parity: ``torchtitan/distributed/expert_parallel.py:26-228``).

Routed experts are sharded ``Shard(0)`` over the ``ep`` mesh (each rank owns
``E / ep`` consecutive experts).  ``ep_dispatch`` replaces the local expert
call of ``MoE``:

  1. all-to-all of per-expert counts (``[ep, E/ep]`` per rank) so every rank
     learns how many rows it receives for each of its experts;
  2. all-to-all of the expert-sorted routed rows (variable split sizes);
  3. rows arrive grouped (source rank, local expert) and are permuted to
     expert-major order, run through the local grouped experts, permuted back;
  4. reverse all-to-all returns each row to the rank that routed it.

Both token all-to-alls are differentiable (the backward is the mirrored
all-to-all).  Split sizes need one device->host copy of the counts, as in the
reference.
"""
from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn as nn
from torch.distributed.nn.functional import all_to_all_single as a2a_autograd


def make_ep_dispatch(ep_group, num_experts: int):
    ep = dist.get_world_size(ep_group)
    if num_experts % ep:
        raise ValueError(f"num_experts {num_experts} not divisible by ep degree {ep}")
    e_local = num_experts // ep

    def dispatch(routed: torch.Tensor, counts: torch.Tensor, experts: nn.Module) -> torch.Tensor:
        send_counts = counts.view(ep, e_local).to(torch.int64).contiguous()
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=ep_group)
        both = torch.stack([send_counts.sum(1), recv_counts.sum(1)]).cpu()
        in_splits, out_splits = both[0].tolist(), both[1].tolist()
        recv = a2a_autograd(routed.new_empty(sum(out_splits), routed.shape[1]), routed.contiguous(),
                            out_splits, in_splits, group=ep_group)
        expert_of_row = torch.repeat_interleave(
            torch.arange(e_local, device=routed.device).repeat(ep), recv_counts.flatten())
        perm = torch.argsort(expert_of_row, stable=True)
        local_counts = recv_counts.sum(0)
        out_sorted = experts(recv[perm], local_counts)
        inv = torch.empty_like(perm)
        inv[perm] = torch.arange(perm.numel(), device=perm.device)
        out = out_sorted[inv]
        return a2a_autograd(out.new_empty(sum(in_splits), out.shape[1]), out.contiguous(), in_splits, out_splits,
                            group=ep_group)

    return dispatch


def apply_ep(moe_modules: list[nn.Module], ep_mesh, backend: str = "standard") -> None:
    """``backend``: ``standard`` = NCCL all-to-all dispatch above; ``fused`` = rows stored
    straight into the owners' padded expert-major buffers over peer memory
    (``parallel.ep_fused``)."""
    from torch.distributed.tensor import Shard, distribute_tensor

    two_d = ep_mesh.ndim == 2  # [ep, etp]: expert dim over ep, hidden dim over etp
    group = ep_mesh["ep"].get_group() if two_d else ep_mesh.get_group()
    for moe in moe_modules:
        ex = moe.experts
        for name, hdim in (("w1", 1), ("w2", 2), ("w3", 1)):
            p = getattr(ex, name)
            place = [Shard(0), Shard(hdim)] if two_d else [Shard(0)]
            setattr(ex, name, nn.Parameter(distribute_tensor(p.data, ep_mesh, place)))
        if backend == "fused":
            from .ep_fused import make_fused_ep_dispatch

            moe.ep_dispatch = make_fused_ep_dispatch(group, moe.num_experts)
        else:
            moe.ep_dispatch = make_ep_dispatch(group, moe.num_experts)
