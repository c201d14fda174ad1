"""Parallelize a Llama 3 model: TP/SP -> CP -> AC -> FSDP2
(order and meshes as in ``models/llama3/parallelize.py:45-140`` of the reference)."""
from __future__ import annotations

from typing import Any

import torch.nn as nn

from torchtitan_b200.config import TORCH_DTYPE_MAP
from torchtitan_b200.parallel.activation_checkpoint import apply_ac
from torchtitan_b200.parallel.context_parallel import apply_cp_to_attention_modules
from torchtitan_b200.parallel.fsdp import (
    dp_mesh,
    apply_fsdp,
    apply_replica_mixed_precision,
    replica_mixed_precision_applicable,
)
from torchtitan_b200.parallel.peer_dp import apply_peer_dp, peer_dp_applicable
from torchtitan_b200.parallel.tensor_parallel import apply_tp_llama, maybe_enable_async_tp
from torchtitan_b200.utils.logging import logger


def parallelize_llama(model: nn.Module, *, parallel_dims: Any, training: Any, model_converters: Any = None,
                      parallelism: Any, compile_config: Any = None, ac_config: Any, dump_folder: str = "",
                      **_: Any) -> nn.Module:
    if training.seq_len % parallel_dims.seq_len_divisor:
        raise ValueError(f"seq_len {training.seq_len} must be divisible by 2*cp*tp = {parallel_dims.seq_len_divisor}")
    if parallel_dims.tp_enabled:
        tp_mesh = parallel_dims.get_mesh("tp")
        apply_tp_llama(model, tp_mesh, loss_parallel=not parallelism.disable_loss_parallel,
                       sequence_parallel=parallelism.enable_sequence_parallel)
        maybe_enable_async_tp(parallelism, tp_mesh)
        logger.info(f"applied tensor parallel (tp={parallel_dims.tp}, sp={parallelism.enable_sequence_parallel})")
    if parallel_dims.cp_enabled:
        apply_cp_to_attention_modules([b.attention for b in model.layers.values()], parallel_dims.get_mesh("cp"),
                                      method=parallelism.context_parallel_method,
                                      load_balance=parallelism.context_parallel_load_balancer == "headtail")
        logger.info(f"applied context parallel ({parallelism.context_parallel_method}, cp={parallel_dims.cp})")
    if ac_config.mode != "none":
        apply_ac(model, ac_config)
        logger.info(f"applied {ac_config.mode} activation checkpointing")
    if peer_dp_applicable(parallel_dims, training, parallelism):
        apply_peer_dp(model, dp_mesh(parallel_dims), bucket_mb=parallelism.data_parallel_bucket_mb)
        logger.info("data parallel: replicated bf16 weights, sharded fp32 optimizer, peer-memory collectives")
    elif replica_mixed_precision_applicable(parallel_dims, training):
        apply_replica_mixed_precision(model)
        logger.info("single replica: bf16 compute weights with fp32 masters in the optimizer (no FSDP wrap)")
    else:
        apply_fsdp(model, dp_mesh(parallel_dims), param_dtype=TORCH_DTYPE_MAP[training.mixed_precision_param],
                   reduce_dtype=TORCH_DTYPE_MAP[training.mixed_precision_reduce],
                   pp_enabled=parallel_dims.pp_enabled, cpu_offload=training.enable_cpu_offload,
                   reshard_after_forward_policy=parallelism.fsdp_reshard_after_forward)
        logger.info("applied FSDP2 (fully_shard) to the model")
    return model
