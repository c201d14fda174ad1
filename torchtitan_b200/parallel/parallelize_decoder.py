"""One parallelize function for the decoder families built from the common
blocks (Qwen3, DeepSeek-V3, Llama 4, GPT-OSS): TP/SP -> CP -> EP -> AC -> DP.

The order and the meshes follow the reference's per-family functions
(``models/llama4/parallelize.py:58-632``, ``models/deepseek_v3/parallelize.py:38-293``,
``models/qwen3/parallelize.py``): tensor parallelism on attention and dense
MLPs, context parallelism on the attention modules (ring or Ulysses), routed
experts sharded over ``ep``, activation checkpointing, then FSDP2 (``efsdp``
mesh for experts) or, for pure data parallelism on one node, the peer-memory
data-parallel runtime.

Blocks are discovered by attribute: ``block.attention`` (any module with a
``cp_hook`` attribute), and either ``block.feed_forward`` (dense SwiGLU) or
``block.moe`` (``models.common.moe.MoE``).
"""
from __future__ import annotations

from typing import Any

import torch.nn as nn

from torchtitan_b200.config import TORCH_DTYPE_MAP
from torchtitan_b200.parallel.activation_checkpoint import apply_ac
from torchtitan_b200.parallel.context_parallel import apply_cp_to_attention_modules
from torchtitan_b200.parallel.expert_parallel import apply_ep
from torchtitan_b200.parallel.fsdp import (
    apply_fsdp,
    apply_replica_mixed_precision,
    dp_mesh,
    replica_mixed_precision_applicable,
)
from torchtitan_b200.parallel.peer_dp import apply_peer_dp, peer_dp_applicable
from torchtitan_b200.utils.logging import logger


def _apply_tp(model: nn.Module, tp_mesh, parallelism: Any, ep_degree: int = 1) -> None:
    from torchtitan_b200.models.common import GQAttention
    from torchtitan_b200.parallel.tensor_parallel import apply_tp_llama, maybe_enable_async_tp

    from torchtitan_b200.models.common.moe import MoE

    sp = parallelism.enable_sequence_parallel
    first = next(iter(model.layers.values()))
    if type(first.attention).__name__ == "GptOssAttention":
        from torchtitan_b200.parallel.tensor_parallel import apply_tp_gpt_oss

        etp = parallelism.expert_tensor_parallel_degree > 1
        if etp and ep_degree > 1:
            raise NotImplementedError("GPT-OSS experts: expert tensor parallelism with expert parallelism is not wired")
        apply_tp_gpt_oss(model, tp_mesh, loss_parallel=not parallelism.disable_loss_parallel, sequence_parallel=sp,
                         etp=etp)
        maybe_enable_async_tp(parallelism, tp_mesh)
        return
    for blk in model.layers.values():
        att = getattr(blk, "attention", None)
        if not isinstance(att, GQAttention) and not hasattr(att, "wkv_a"):
            raise NotImplementedError(f"{type(model).__name__}: tensor parallelism covers GQA and MLA attention")
        moe = getattr(blk, "moe", None)
        if moe is not None and not isinstance(moe, MoE):
            raise NotImplementedError(f"tensor parallelism for {type(moe).__name__} is not wired")
    apply_tp_llama(model, tp_mesh, loss_parallel=not parallelism.disable_loss_parallel, sequence_parallel=sp)
    group = tp_mesh.get_group()
    etp = parallelism.expert_tensor_parallel_degree
    if etp not in (1, tp_mesh.size()):
        raise ValueError(f"expert_tensor_parallel_degree must be 1 or the TP degree ({tp_mesh.size()})")
    for blk in model.layers.values():
        moe = getattr(blk, "moe", None)
        if moe is not None and etp > 1:
            from torchtitan_b200.parallel.tensor_parallel import apply_etp

            apply_etp(moe, tp_mesh, sp, distribute_experts=ep_degree == 1)
        elif moe is not None and sp:
            # routed tokens are this rank's sequence shard; experts, router and shared experts are
            # replicated over TP, so their weight gradients are summed over TP
            moe.experts.grad_reduce_group = group
            moe.router.gate.grad_reduce_group = group
            if moe.shared_experts is not None:
                for lin in (moe.shared_experts.w1, moe.shared_experts.w2, moe.shared_experts.w3):
                    lin.grad_reduce_group = group
            moe.tp_count_group = group  # token counts for the load-balancing bias cover all TP shards
    maybe_enable_async_tp(parallelism, tp_mesh)


def parallelize_decoder(model: nn.Module, *, parallel_dims: Any, training: Any, parallelism: Any, ac_config: Any,
                        model_converters: Any = None, compile_config: Any = None, dump_folder: str = "",
                        **_: Any) -> nn.Module:
    pd = parallel_dims
    if training.seq_len % pd.seq_len_divisor:
        raise ValueError(f"seq_len {training.seq_len} must be divisible by 2*cp*tp = {pd.seq_len_divisor}")
    if pd.tp_enabled:
        _apply_tp(model, pd.get_mesh("tp"), parallelism, pd.ep)
        logger.info(f"applied tensor parallel (tp={pd.tp})")
    if pd.cp_enabled:
        attns = [blk.attention for blk in model.layers.values()]
        apply_cp_to_attention_modules(attns, pd.get_mesh("cp"), method=parallelism.context_parallel_method,
                                      load_balance=parallelism.context_parallel_load_balancer == "headtail")
        logger.info(f"applied context parallel ({parallelism.context_parallel_method}, cp={pd.cp})")
    moes = [blk.moe for blk in model.layers.values() if getattr(blk, "moe", None) is not None]
    if pd.ep_enabled and moes:
        # with expert tensor parallelism the experts are sharded over [ep, etp] together
        mesh = pd.get_mesh(["ep", "etp"]) if pd.etp_enabled else pd.get_mesh("ep")
        apply_ep(moes, mesh, backend=parallelism.expert_parallel_comm_backend)
        logger.info(f"applied expert parallel (ep={pd.ep}) to {len(moes)} MoE layers")
    if ac_config.mode != "none":
        apply_ac(model, ac_config)
        logger.info(f"applied {ac_config.mode} activation checkpointing")
    if peer_dp_applicable(pd, training, parallelism):
        return apply_peer_dp(model, dp_mesh(pd), bucket_mb=parallelism.data_parallel_bucket_mb)
    if replica_mixed_precision_applicable(pd, training):
        return apply_replica_mixed_precision(model)
    apply_fsdp(model, dp_mesh(pd), param_dtype=TORCH_DTYPE_MAP[training.mixed_precision_param],
               reduce_dtype=TORCH_DTYPE_MAP[training.mixed_precision_reduce], pp_enabled=pd.pp_enabled,
               cpu_offload=training.enable_cpu_offload,
               reshard_after_forward_policy=parallelism.fsdp_reshard_after_forward,
               ep_degree=pd.ep, edp_mesh=pd.get_mesh("efsdp") if pd.ep_enabled else None)
    return model
