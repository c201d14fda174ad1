"""Kimi-Linear family: flavors and ``ModelSpec`` registry
(parity: ``experiments/attention_residual/kimi_linear/__init__.py:76-126`` and
``config_registry.py:61-412``).

Flavors: the scaling-law sweep sizes ``194m, 241m, 296m, 436m, 528m,
447m_aligned`` and ``48b`` (48B-A3B: 27 layers, MLA at 4,8,...,24,27,
256 experts), each as ``<size>_baseline``, ``<size>_block_attn_res`` (8
AttnRes blocks) and ``<size>_full_attn_res`` (one block per layer), plus a
tiny ``debugmodel`` for tests.
"""
from __future__ import annotations

import copy

from torchtitan_b200.components.loss import build_cross_entropy_loss
from torchtitan_b200.components.optimizer import build_optimizers_with_moe_load_balancing
from torchtitan_b200.parallel.pipeline import pipeline_llm
from torchtitan_b200.protocols import ModelSpec

from .model import KimiLinearModel, KimiLinearModelArgs
from .parallelize import parallelize_kimi
from .state_dict_adapter import KimiLinearStateDictAdapter

# name: (n_layers, heads, d_model, d_ff per expert)  -- Kimi Linear tech report scaling sweep
_SWEEP = {
    "194m": (12, 12, 896, 400),
    "241m": (13, 13, 960, 432),
    "296m": (14, 14, 1024, 464),
    "436m": (16, 16, 1168, 528),
    "528m": (17, 17, 1264, 560),
    "447m_aligned": (16, 16, 1024, 768),
    "48b": (27, 32, 2304, 1024),
}
_48B_MLA = [4, 8, 12, 16, 20, 24, 27]


def _kda_mla_layers(n: int, ratio: int = 3) -> tuple[list[int], list[int]]:
    kda, mla = [], []
    for i in range(1, n + 1):
        (mla if i % (ratio + 1) == 0 else kda).append(i)
    return kda, mla


def build_args(size: str, *, num_experts: int | None = None, attn_res_blocks: int = 0,
               vocab_size: int = 163840) -> KimiLinearModelArgs:
    if size == "debugmodel":
        return KimiLinearModelArgs(vocab_size=2048, hidden_size=256, num_hidden_layers=4, intermediate_size=512,
                                   num_attention_heads=4, kv_lora_rank=64, qk_nope_head_dim=64,
                                   qk_rope_head_dim=64, v_head_dim=128, kda_num_heads=4, kda_head_dim=64,
                                   kda_layers=[1, 2, 3], full_attn_layers=[4], num_experts=8,
                                   num_experts_per_token=2, moe_intermediate_size=128, use_grouped_topk=False,
                                   tie_word_embeddings=False, attn_res_blocks=attn_res_blocks)
    L, H, d, dff = _SWEEP[size]
    if size == "48b":
        mla = list(_48B_MLA)
        kda = [i for i in range(1, L + 1) if i not in mla]
        kw = dict(kv_lora_rank=512, qk_nope_head_dim=128, qk_rope_head_dim=64, v_head_dim=128, kda_head_dim=128,
                  intermediate_size=9216, tie_word_embeddings=False, use_grouped_topk=True)
        experts = 256
    else:
        kda, mla = _kda_mla_layers(L)
        if size.endswith("_aligned"):
            nope = max(32, (d // H) & ~15)
            lora = (d // 2) & ~63
        else:
            nope = max(32, d // H)
            lora = d // 2
        kw = dict(kv_lora_rank=lora, qk_nope_head_dim=nope, qk_rope_head_dim=max(16, nope // 2), v_head_dim=nope,
                  kda_head_dim=nope, intermediate_size=dff, tie_word_embeddings=True, use_grouped_topk=False)
        experts = 32
    return KimiLinearModelArgs(vocab_size=vocab_size, hidden_size=d, num_hidden_layers=L, num_attention_heads=H,
                               kda_num_heads=H, kda_layers=kda, full_attn_layers=mla,
                               num_experts=num_experts or experts, moe_intermediate_size=dff,
                               attn_res_blocks=attn_res_blocks, **kw)


def _flavors() -> dict[str, KimiLinearModelArgs]:
    out = {"debugmodel": build_args("debugmodel"),
           "debugmodel_block_attn_res": build_args("debugmodel", attn_res_blocks=2)}
    for size, (L, *_rest) in _SWEEP.items():
        out[f"{size}_baseline"] = build_args(size)
        out[f"{size}_block_attn_res"] = build_args(size, attn_res_blocks=min(8, L))
        out[f"{size}_full_attn_res"] = build_args(size, attn_res_blocks=L)
    return out


kimi_linear_args = _flavors()


def model_registry(flavor: str) -> ModelSpec:
    if flavor not in kimi_linear_args:
        raise ValueError(f"unknown kimi_linear flavor '{flavor}', available: {sorted(kimi_linear_args)}")
    return ModelSpec(
        name="kimi_linear",
        flavor=flavor,
        model=copy.deepcopy(kimi_linear_args[flavor]),
        parallelize_fn=parallelize_kimi,
        pipelining_fn=pipeline_llm,
        build_loss_fn=build_cross_entropy_loss,
        post_optimizer_build_fn=build_optimizers_with_moe_load_balancing,
        state_dict_adapter=KimiLinearStateDictAdapter,
    )


__all__ = ["KimiLinearModel", "KimiLinearModelArgs", "model_registry", "kimi_linear_args", "build_args"]
