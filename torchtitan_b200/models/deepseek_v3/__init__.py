"""DeepSeek-V3 family: flavors and the ``ModelSpec`` registry (parity: reference
``models/deepseek_v3/__init__.py``; 16B = DeepSeek-V2-Lite shape, 236B = V2, 671B = V3)."""
from __future__ import annotations

import copy

from torchtitan_b200.components.loss import build_cross_entropy_loss
from torchtitan_b200.parallel.parallelize_decoder import parallelize_decoder
from torchtitan_b200.parallel.pipeline import pipeline_llm
from torchtitan_b200.protocols import ModelSpec

from .model import DeepSeekV3Model, DeepSeekV3ModelArgs
from .state_dict_adapter import DeepSeekV3StateDictAdapter

A = DeepSeekV3ModelArgs
deepseekv3_args = {
    "debugmodel": A(vocab_size=2048, dim=256, inter_dim=1024, moe_inter_dim=256, n_layers=6, n_dense_layers=1,
                    n_heads=16, n_routed_experts=8, n_shared_experts=2, n_activated_experts=3, mscale=0.70),
    "debugmodel_qlora": A(vocab_size=2048, dim=256, inter_dim=1024, moe_inter_dim=256, n_layers=4,
                          n_dense_layers=1, n_heads=16, n_routed_experts=8, n_shared_experts=1,
                          n_activated_experts=2, n_expert_groups=4, n_limited_groups=2, score_func="sigmoid",
                          route_norm=True, route_scale=2.5, q_lora_rank=128, mscale=0.70),
    "16B": A(vocab_size=102400, dim=2048, inter_dim=10944, moe_inter_dim=1408, n_layers=27, n_dense_layers=1,
             n_heads=16, n_routed_experts=64, n_shared_experts=2, n_activated_experts=6, mscale=0.707),
    "236B": A(vocab_size=102400, dim=5120, inter_dim=12288, moe_inter_dim=1536, n_layers=60, n_dense_layers=1,
              n_heads=128, n_routed_experts=160, n_shared_experts=2, n_activated_experts=6, n_expert_groups=8,
              n_limited_groups=3, route_scale=16.0, q_lora_rank=1536),
    "671B": A(vocab_size=129280, dim=7168, inter_dim=18432, moe_inter_dim=2048, n_layers=61, n_dense_layers=3,
              n_heads=128, n_routed_experts=256, n_shared_experts=1, n_activated_experts=8, n_expert_groups=8,
              n_limited_groups=4, score_func="sigmoid", route_norm=True, route_scale=2.5, q_lora_rank=1536),
}


def model_registry(flavor: str) -> ModelSpec:
    if flavor not in deepseekv3_args:
        raise ValueError(f"unknown deepseek_v3 flavor '{flavor}', available: {sorted(deepseekv3_args)}")
    from torchtitan_b200.components.optimizer import build_optimizers_with_moe_load_balancing

    return ModelSpec(name="deepseek_v3", flavor=flavor, model=copy.deepcopy(deepseekv3_args[flavor]),
                     parallelize_fn=parallelize_decoder, pipelining_fn=pipeline_llm,
                     build_loss_fn=build_cross_entropy_loss,
                     post_optimizer_build_fn=build_optimizers_with_moe_load_balancing,
                     state_dict_adapter=DeepSeekV3StateDictAdapter)


__all__ = ["DeepSeekV3Model", "DeepSeekV3ModelArgs", "model_registry", "deepseekv3_args"]
