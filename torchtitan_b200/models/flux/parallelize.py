"""Parallelism for FLUX (parity: reference ``models/flux/parallelize.py``): context
parallelism (Ulysses: every rank holds a slice of the text and image tokens; attention
trades it for all tokens of a head slice), activation checkpointing per double/single
stream block, then FSDP2 (or HSDP) over the data-parallel and context-parallel ranks
with one sharding unit per block plus the root.  Tensor, pipeline and expert
parallelism are not wired for this family."""
from __future__ import annotations

from typing import Any

import torch.nn as nn
from torch.distributed.fsdp import CPUOffloadPolicy, MixedPrecisionPolicy, fully_shard

from torchtitan_b200.config import TORCH_DTYPE_MAP
from torchtitan_b200.parallel import fsdp as _fsdp
from torchtitan_b200.parallel.activation_checkpoint import apply_ac


def parallelize_flux(model: nn.Module, *, parallel_dims: Any, training: Any, parallelism: Any, ac_config: Any,
                     **_: Any) -> nn.Module:
    pd = parallel_dims
    if pd.tp_enabled or pd.pp_enabled or pd.ep_enabled:
        raise NotImplementedError("flux: data, context parallelism and activation checkpointing are wired")
    if pd.cp_enabled:
        if model.model_args.num_heads % pd.cp:
            raise ValueError(f"flux: cp degree {pd.cp} must divide num_heads {model.model_args.num_heads}")
        group = pd.get_mesh("cp").get_group()
        for blk in list(model.double_blocks) + list(model.single_blocks):
            blk.cp_group = group
    model.ac_block_containers = [model.double_blocks, model.single_blocks]
    apply_ac(model, ac_config)
    if not (pd.dp_enabled or pd.cp_enabled):
        return model
    import torch.distributed as dist

    mesh = _fsdp.dp_mesh(pd)
    _fsdp._GLOO = dist.is_initialized() and dist.get_backend() == "gloo"
    model._fsdp_grad_compensation = mesh.size() if _fsdp._GLOO else 1
    mp = MixedPrecisionPolicy(param_dtype=TORCH_DTYPE_MAP[training.mixed_precision_param],
                              reduce_dtype=TORCH_DTYPE_MAP[training.mixed_precision_reduce])
    cfg: dict[str, Any] = {"mesh": mesh, "mp_policy": mp}
    if training.enable_cpu_offload:
        cfg["offload_policy"] = CPUOffloadPolicy()
    reshard = parallelism.fsdp_reshard_after_forward != "never"
    blocks = list(model.double_blocks) + list(model.single_blocks)
    for i, blk in enumerate(blocks):
        _fsdp._disable_grad_division(fully_shard(blk, **cfg, reshard_after_forward=reshard and i < len(blocks) - 1))
    _fsdp._disable_grad_division(fully_shard(model, **cfg))
    return model
