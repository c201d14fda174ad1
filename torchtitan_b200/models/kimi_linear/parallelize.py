"""Parallelize Kimi-Linear: Ulysses CP -> EP -> AC -> FSDP2
(reference: ``kimi_linear/parallelize.py:73-1076``; Ulysses CP is new here,
the reference raises NotImplementedError for CP on Kimi).

* Ulysses CP: MLA layers all-to-all q/k/v sequence<->heads around the
  attention kernel; KDA layers all-to-all their per-head streams so the short
  convolution and the recurrence see the full sequence for H/cp heads.
* EP: routed experts ``Shard(0)`` over ``ep``; dispatch/combine all-to-alls.
* FSDP2 over ``fsdp`` for dense params, over ``efsdp`` for routed experts.
"""
from __future__ import annotations

from typing import Any

import torch.nn as nn

from torchtitan_b200.config import TORCH_DTYPE_MAP
from torchtitan_b200.parallel.activation_checkpoint import apply_ac
from torchtitan_b200.parallel.context_parallel import ulysses_hook
from torchtitan_b200.parallel.expert_parallel import apply_ep
from torchtitan_b200.parallel.fsdp import (
    dp_mesh,
    apply_fsdp,
    apply_replica_mixed_precision,
    replica_mixed_precision_applicable,
)
from torchtitan_b200.utils.logging import logger


def parallelize_kimi(model: nn.Module, *, parallel_dims: Any, training: Any, parallelism: Any, ac_config: Any,
                     model_converters: Any = None, compile_config: Any = None, dump_folder: str = "",
                     **_: Any) -> nn.Module:
    pd = parallel_dims
    if pd.tp_enabled:
        from torchtitan_b200.parallel.tensor_parallel import apply_tp_kimi

        if model.model_args.tie_word_embeddings:
            raise NotImplementedError("tensor parallelism with tied embeddings is not wired")
        apply_tp_kimi(model, pd.get_mesh("tp"), loss_parallel=not parallelism.disable_loss_parallel)
        logger.info(f"applied tensor parallel to MLA heads and dense MLPs (tp={pd.tp})")
    if pd.cp_enabled:
        if parallelism.context_parallel_method != "ulysses":
            raise ValueError("Kimi-Linear context parallelism uses Ulysses (KDA needs the whole sequence per head)")
        group = pd.get_mesh("cp").get_group()
        for blk in model.layers.values():
            if blk.is_linear_attn:
                if blk.self_attn.h % pd.cp:
                    raise ValueError("cp must divide kda_num_heads")
                blk.self_attn.cp_group = group
            else:
                blk.self_attn.cp_hook = ulysses_hook(group)
        logger.info(f"applied Ulysses context parallel (cp={pd.cp})")
    moes = [blk.moe for blk in model.layers.values() if getattr(blk, "moe", None) is not None]
    if pd.ep_enabled and moes:
        apply_ep(moes, pd.get_mesh("ep"), backend=parallelism.expert_parallel_comm_backend)
        logger.info(f"applied expert parallel (ep={pd.ep}) to {len(moes)} MoE layers")
    if ac_config.mode != "none":
        apply_ac(model, ac_config)
    if replica_mixed_precision_applicable(pd, training):
        return apply_replica_mixed_precision(model)
    apply_fsdp(model, dp_mesh(pd), param_dtype=TORCH_DTYPE_MAP[training.mixed_precision_param],
               reduce_dtype=TORCH_DTYPE_MAP[training.mixed_precision_reduce], pp_enabled=pd.pp_enabled,
               cpu_offload=training.enable_cpu_offload,
               reshard_after_forward_policy=parallelism.fsdp_reshard_after_forward,
               ep_degree=pd.ep, edp_mesh=pd.get_mesh("efsdp") if pd.ep_enabled else None)
    return model
