"""FSDP2 / HSDP application (parity: ``models/llama3/parallelize.py:244-324``).

Each transformer block, the embedding, and ``[norm, output]`` become FSDP2
units on the ``fsdp`` (or ``[dp_replicate, fsdp]`` for HSDP) mesh with
``MixedPrecisionPolicy(param=bf16, reduce=fp32)``.  Gradient division by the
DP size is disabled: the loss is already normalised by the global token
count.  Reshard-after-forward: ``default`` = yes except the last block (whose
parameters are needed immediately by backward) and never under PP.
"""
from __future__ import annotations

from typing import Any

import torch
import torch.nn as nn
from torch.distributed.fsdp import CPUOffloadPolicy, MixedPrecisionPolicy, fully_shard


_GLOO = False


def _disable_grad_division(m) -> None:
    # gloo has no PREMUL_SUM: keep FSDP's mean there and let the trainer scale
    # the backward seed by the DP size instead (model._fsdp_grad_compensation)
    # (fully_shard of a list of modules returns the list: each is an FSDP module)
    for mod in (m if isinstance(m, (list, tuple)) else [m]):
        if not _GLOO and hasattr(mod, "set_gradient_divide_factor"):
            mod.set_gradient_divide_factor(1.0)


def _local_tensor_mode_active() -> bool:
    try:
        from torch.distributed._local_tensor import local_tensor_mode
    except ImportError:
        return False
    return local_tensor_mode() is not None


def apply_fsdp(model: nn.Module, dp_mesh: Any, *, param_dtype: torch.dtype, reduce_dtype: torch.dtype,
               pp_enabled: bool = False, cpu_offload: bool = False, reshard_after_forward_policy: str = "default",
               ep_degree: int = 1, edp_mesh: Any = None) -> nn.Module:
    if _local_tensor_mode_active():
        # FSDP2 frees and regrows parameter storage, which LocalTensor (one process simulating
        # every rank) does not have: a data-parallel mesh of one needs no wrap there
        if dp_mesh is None or dp_mesh.size() == 1:
            return model
        raise NotImplementedError("comm.mode=local_tensor with FSDP (dp_shard > 1): torch's FSDP2 cannot resize "
                                  "LocalTensor storage; simulate TP/CP/PP meshes with dp_shard = 1 or use gloo ranks")
    # forward inputs are not cast: activations are already in the param dtype
    # (bf16 embedding output) and the fp32 RoPE tables must stay fp32
    mp = MixedPrecisionPolicy(param_dtype=param_dtype, reduce_dtype=reduce_dtype, cast_forward_inputs=False)
    cfg: dict[str, Any] = {"mesh": dp_mesh, "mp_policy": mp}
    if cpu_offload:
        cfg["offload_policy"] = CPUOffloadPolicy()
    if reshard_after_forward_policy == "always":
        reshard = True
    elif reshard_after_forward_policy == "never":
        reshard = False
    elif reshard_after_forward_policy == "default":
        reshard = not pp_enabled
    else:
        raise ValueError(f"invalid reshard_after_forward_policy {reshard_after_forward_policy}")

    global _GLOO
    import torch.distributed as dist

    _GLOO = dist.is_initialized() and dist.get_backend() == "gloo"
    model._fsdp_grad_compensation = dp_mesh.size() if _GLOO else 1
    for unit in getattr(model, "fsdp_extra_units", ()):  # e.g. vision encoder blocks
        _disable_grad_division(fully_shard(unit, **cfg, reshard_after_forward=reshard))
    first = getattr(model, "pp_first_module", "tok_embeddings")
    if getattr(model, first, None) is not None:
        _disable_grad_division(fully_shard(getattr(model, first), **cfg, reshard_after_forward=reshard))
    layers = [l for l in model.layers.values() if l is not None]
    for i, block in enumerate(layers):
        # routed experts are sharded on the expert-data-parallel mesh
        moe = getattr(block, "moe", None) or getattr(getattr(block, "ffn", None), "_moe", None)
        if moe is not None and ep_degree > 1 and edp_mesh is not None:
            ecfg = dict(cfg, mesh=edp_mesh)
            if _GLOO:  # experts average over efsdp, the compensated loss assumed the dp mesh
                moe.experts.grad_scale = edp_mesh.size() / dp_mesh.size()
            _disable_grad_division(fully_shard(moe.experts, **ecfg, reshard_after_forward=reshard))
        last = i == len(layers) - 1
        _disable_grad_division(
            fully_shard(block, **cfg, reshard_after_forward=reshard and not last)
        )
    last = getattr(model, "pp_last_modules", ("norm", "output"))
    tail = [getattr(model, n) for n in last if getattr(model, n, None) is not None]
    if tail:
        _disable_grad_division(fully_shard(tail, **cfg, reshard_after_forward=False))
    _disable_grad_division(fully_shard(model, **cfg))
    return model


def dp_mesh_names(parallel_dims) -> list[str]:
    """Mesh dims that data-parallel gradient reduction spans: ``dp_replicate`` is left out
    when it holds semi-synchronous replicas (LocalSGD / DiLoCo), which reduce nothing
    between their synchronisations."""
    if parallel_dims.dp_replicate_enabled and not getattr(parallel_dims, "semi_sync_replicas", False):
        return ["dp_replicate", "fsdp"]
    return ["fsdp"]


def dp_mesh(parallel_dims):
    names = dp_mesh_names(parallel_dims)
    return parallel_dims.get_mesh(names if len(names) > 1 else names[0])


def apply_ddp(model: nn.Module, dp_mesh: Any) -> nn.Module:
    """Pure data parallel: replicate via FSDP2 on the replicate mesh."""
    return apply_fsdp(model, dp_mesh, param_dtype=torch.bfloat16, reduce_dtype=torch.float32)


def replica_mixed_precision_applicable(parallel_dims, training) -> bool:
    """One data-parallel rank and nothing to shard: FSDP2 would only add cast/copy traffic."""
    return (torch.cuda.is_available() and parallel_dims.world_size == 1 and not parallel_dims.pp_enabled
            and training.mixed_precision_param == "bfloat16" and training.dtype == "float32"
            and not training.enable_cpu_offload)


def apply_replica_mixed_precision(model: nn.Module) -> nn.Module:
    """Mark ``model`` for single-replica mixed precision: after weight init the
    trainer calls ``materialize_replica_mixed_precision`` which keeps an fp32
    master copy of every parameter (``param._master``) and turns the parameter
    itself into the bf16 compute weight.  The fused AdamW updates the master
    and rewrites the bf16 weight in the same kernel pass."""
    model._replica_param_dtype = torch.bfloat16
    return model


@torch.no_grad()
def materialize_replica_mixed_precision(model: nn.Module) -> None:
    dt = getattr(model, "_replica_param_dtype", None)
    if dt is None:
        return
    seen = set()
    for p in model.parameters():
        if id(p) in seen or p.dtype != torch.float32:
            continue
        seen.add(id(p))
        master = p.data.clone()
        p.data = p.data.to(dt)
        p._master = master
