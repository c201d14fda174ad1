"""Parallelism for the Llama 3 + SigLIP2 VLM (parity: reference
``experiments/vlm/infra/parallelize.py``): the decoder through the shared decoder path,
each encoder block and the projector as their own FSDP units; tensor parallelism on
the decoder without sequence parallelism (image features are spliced into the full
sequence; the encoder runs replicated on the tensor-parallel ranks)."""
from __future__ import annotations

from typing import Any

import torch.nn as nn

from torchtitan_b200.parallel.parallelize_decoder import parallelize_decoder


def parallelize_vlm(model: nn.Module, *, parallel_dims: Any, parallelism: Any, **kw: Any) -> nn.Module:
    pd = parallel_dims
    if pd.cp_enabled or pd.pp_enabled:
        raise NotImplementedError("vlm: context and pipeline parallelism are not wired")
    if pd.tp_enabled and parallelism.enable_sequence_parallel:
        raise ValueError("vlm: tensor parallelism runs without sequence parallelism "
                         "(set --parallelism.no-enable-sequence-parallel)")
    model.fsdp_extra_units = list(model.encoder.layers) + [model.projector]
    return parallelize_decoder(model, parallel_dims=pd, parallelism=parallelism, **kw)
