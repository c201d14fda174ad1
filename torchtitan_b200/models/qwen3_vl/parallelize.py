"""Parallelism for Qwen3-VL (parity: reference ``models/qwen3_vl/parallelize.py``).

The decoder goes through the shared decoder path (TP -> EP -> AC -> FSDP2 or the
peer-memory data-parallel runtime).  Under FSDP2 every vision block and the mergers are
their own sharding units (``fsdp_extra_units``).  Tensor parallelism covers the
decoder only, without sequence parallelism: the vision tokens are spliced into the
full sequence, and the encoder runs replicated on every tensor-parallel rank (same
inputs, same gradients).  Context and pipeline parallelism are not wired for this
family.
"""
from __future__ import annotations

from typing import Any

import torch.nn as nn

from torchtitan_b200.parallel.parallelize_decoder import parallelize_decoder


def parallelize_qwen3_vl(model: nn.Module, *, parallel_dims: Any, parallelism: Any, **kw: Any) -> nn.Module:
    pd = parallel_dims
    if pd.cp_enabled or pd.pp_enabled:
        raise NotImplementedError("qwen3_vl: context and pipeline parallelism are not wired")
    if pd.tp_enabled and parallelism.enable_sequence_parallel:
        raise ValueError("qwen3_vl: tensor parallelism runs without sequence parallelism "
                         "(set --parallelism.enable-sequence-parallel false)")
    ve = model.vision_encoder
    model.fsdp_extra_units = list(ve.blocks) + [ve.merger, *ve.deepstack_mergers]
    return parallelize_decoder(model, parallel_dims=pd, parallelism=parallelism, **kw)
