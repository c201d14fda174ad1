"""Qwen3 family: flavors and the ``ModelSpec`` registry (parity: reference
``models/qwen3/__init__.py``; sizes from the published Qwen3 configs)."""
from __future__ import annotations

import copy

from torchtitan_b200.components.loss import build_cross_entropy_loss
from torchtitan_b200.parallel.parallelize_decoder import parallelize_decoder
from torchtitan_b200.parallel.pipeline import pipeline_llm
from torchtitan_b200.protocols import ModelSpec

from .model import Qwen3Model, Qwen3ModelArgs
from .state_dict_adapter import Qwen3StateDictAdapter

A = Qwen3ModelArgs
qwen3_args = {
    "debugmodel": A(dim=256, n_layers=8, n_heads=16, n_kv_heads=8, head_dim=128, hidden_dim=3072, vocab_size=2048,
                    max_seq_len=4096),
    "debugmodel_moe": A(dim=256, n_layers=8, n_heads=16, n_kv_heads=8, head_dim=128, hidden_dim=3072,
                        vocab_size=2048, max_seq_len=4096, moe_enabled=True, num_experts=8, top_k=2,
                        moe_hidden_dim=256),
    "0.6B": A(dim=1024, n_layers=28, n_heads=16, n_kv_heads=8, hidden_dim=3072, enable_weight_tying=True),
    "1.7B": A(dim=2048, n_layers=28, n_heads=16, n_kv_heads=8, hidden_dim=6144, enable_weight_tying=True),
    "4B": A(dim=2560, n_layers=36, n_heads=32, n_kv_heads=8, hidden_dim=9728, enable_weight_tying=True),
    "8B": A(dim=4096, n_layers=36, n_heads=32, n_kv_heads=8, hidden_dim=12288),
    "14B": A(dim=5120, n_layers=40, n_heads=40, n_kv_heads=8, hidden_dim=17408),
    "32B": A(dim=5120, n_layers=64, n_heads=64, n_kv_heads=8, hidden_dim=25600),
    "30B-A3B": A(dim=2048, n_layers=48, n_heads=32, n_kv_heads=4, hidden_dim=6144, moe_enabled=True,
                 num_experts=128, top_k=8, moe_hidden_dim=768),
    "235B-A22B": A(dim=4096, n_layers=94, n_heads=64, n_kv_heads=4, hidden_dim=12288, moe_enabled=True,
                   num_experts=128, top_k=8, moe_hidden_dim=1536),
}


def model_registry(flavor: str) -> ModelSpec:
    if flavor not in qwen3_args:
        raise ValueError(f"unknown qwen3 flavor '{flavor}', available: {sorted(qwen3_args)}")
    from torchtitan_b200.components.optimizer import build_optimizers_with_moe_load_balancing

    a = copy.deepcopy(qwen3_args[flavor])
    return ModelSpec(name="qwen3", flavor=flavor, model=a, parallelize_fn=parallelize_decoder,
                     pipelining_fn=pipeline_llm, build_loss_fn=build_cross_entropy_loss,
                     post_optimizer_build_fn=build_optimizers_with_moe_load_balancing if a.moe_enabled else None,
                     state_dict_adapter=Qwen3StateDictAdapter)


__all__ = ["Qwen3Model", "Qwen3ModelArgs", "model_registry", "qwen3_args"]
