"""Qwen3-VL family: flavors and the ``ModelSpec`` registry (parity: reference
``models/qwen3_vl/__init__.py``; sizes from the published Qwen3-VL configs).
The debug flavors use a 2048-token vocabulary with the vision placeholders at its
top, like the other debug models of this framework."""
from __future__ import annotations

import copy

from torchtitan_b200.components.loss import build_cross_entropy_loss
from torchtitan_b200.protocols import ModelSpec

from .model import Qwen3VLModel, Qwen3VLModelArgs, mrope_positions
from .parallelize import parallelize_qwen3_vl
from .state_dict_adapter import Qwen3VLStateDictAdapter

A = Qwen3VLModelArgs
_debug_vision = dict(vision_dim=256, vision_ffn_dim=512, vision_layers=4, vision_heads=4, patch_size=16,
                     num_position_embeddings=1024, deepstack_indices=(1, 2, 3), mrope_section=(8, 8, 8),
                     vocab_size=2048, image_token_id=2046, video_token_id=2047, rope_theta=1000000.0,
                     max_seq_len=4096)
_vit_400m = dict(vision_dim=1024, vision_ffn_dim=4096, vision_layers=24, vision_heads=16,
                 num_position_embeddings=2304, deepstack_indices=(5, 11, 17))
_vit_600m = dict(vision_dim=1152, vision_ffn_dim=4304, vision_layers=27, vision_heads=16,
                 num_position_embeddings=2304, deepstack_indices=(8, 16, 24))
qwen3_vl_args = {
    "debugmodel": A(dim=256, n_layers=4, n_heads=4, n_kv_heads=2, head_dim=64, hidden_dim=512, **_debug_vision),
    "debugmodel_moe": A(dim=256, n_layers=1, n_heads=4, n_kv_heads=2, head_dim=64, hidden_dim=512,
                        moe_enabled=True, num_experts=64, top_k=8, moe_hidden_dim=768, **_debug_vision),
    "2B": A(dim=2048, n_layers=28, n_heads=16, n_kv_heads=8, head_dim=128, hidden_dim=6144,
            enable_weight_tying=True, **_vit_400m),
    "8B": A(dim=4096, n_layers=36, n_heads=32, n_kv_heads=8, head_dim=128, hidden_dim=12288, **_vit_600m),
    "30B-A3B": A(dim=2048, n_layers=48, n_heads=32, n_kv_heads=4, head_dim=128, hidden_dim=6144, moe_enabled=True,
                 num_experts=128, top_k=8, moe_hidden_dim=768, **_vit_600m),
    "235B-A22B": A(dim=4096, n_layers=94, n_heads=64, n_kv_heads=4, head_dim=128, hidden_dim=12288,
                   moe_enabled=True, num_experts=128, top_k=8, moe_hidden_dim=1536, **_vit_600m),
}


def model_registry(flavor: str) -> ModelSpec:
    if flavor not in qwen3_vl_args:
        raise ValueError(f"unknown qwen3_vl flavor '{flavor}', available: {sorted(qwen3_vl_args)}")
    from torchtitan_b200.components.optimizer import build_optimizers_with_moe_load_balancing

    a = copy.deepcopy(qwen3_vl_args[flavor])
    return ModelSpec(name="qwen3_vl", flavor=flavor, model=a, parallelize_fn=parallelize_qwen3_vl,
                     pipelining_fn=None, build_loss_fn=build_cross_entropy_loss,
                     post_optimizer_build_fn=build_optimizers_with_moe_load_balancing if a.moe_enabled else None,
                     state_dict_adapter=Qwen3VLStateDictAdapter)


__all__ = ["Qwen3VLModel", "Qwen3VLModelArgs", "model_registry", "mrope_positions", "qwen3_vl_args"]
