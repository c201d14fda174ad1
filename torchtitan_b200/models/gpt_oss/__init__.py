"""GPT-OSS family: flavors and the ``ModelSpec`` registry (parity: reference
``models/gpt_oss/__init__.py``; 20B and 120B shapes from the published configs)."""
from __future__ import annotations

import copy

from torchtitan_b200.components.loss import build_cross_entropy_loss
from torchtitan_b200.parallel.parallelize_decoder import parallelize_decoder
from torchtitan_b200.parallel.pipeline import pipeline_llm
from torchtitan_b200.protocols import ModelSpec

from .model import GptOssModel, GptOssModelArgs
from .state_dict_adapter import GptOssStateDictAdapter

A = GptOssModelArgs
gptoss_args = {
    "debugmodel": A(vocab_size=2048, dim=256, n_layers=4, n_heads=8, n_kv_heads=2, head_dim=64, num_experts=8,
                    top_k=2, moe_inter_dim=256, sliding_window=64, max_seq_len=4096),
    "20b": A(n_layers=24, num_experts=32),
    "120b": A(n_layers=36, num_experts=128),
}


def model_registry(flavor: str) -> ModelSpec:
    if flavor not in gptoss_args:
        raise ValueError(f"unknown gpt_oss flavor '{flavor}', available: {sorted(gptoss_args)}")
    return ModelSpec(name="gpt_oss", flavor=flavor, model=copy.deepcopy(gptoss_args[flavor]),
                     parallelize_fn=parallelize_decoder, pipelining_fn=pipeline_llm,
                     build_loss_fn=build_cross_entropy_loss, state_dict_adapter=GptOssStateDictAdapter)


__all__ = ["GptOssModel", "GptOssModelArgs", "model_registry", "gptoss_args"]
