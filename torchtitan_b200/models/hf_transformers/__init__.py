"""Hugging Face ``transformers`` modeling backend: flavors and ``ModelSpec`` registry."""
from __future__ import annotations

import copy
from typing import Any

import torch.nn as nn

from torchtitan_b200.components.loss import build_cross_entropy_loss
from torchtitan_b200.protocols import ModelSpec

from .model import HFCausalLM, HFModelArgs

_DEBUG = dict(vocab_size=2048, hidden_size=256, intermediate_size=512, num_hidden_layers=4, num_attention_heads=8,
              num_key_value_heads=4, max_position_embeddings=4096, tie_word_embeddings=False)

hf_args = {
    "llama_debugmodel": HFModelArgs(model_type="llama", config_kwargs=dict(_DEBUG)),
    "qwen3_debugmodel": HFModelArgs(model_type="qwen3", config_kwargs=dict(_DEBUG, head_dim=32)),
    "mistral_debugmodel": HFModelArgs(model_type="mistral", config_kwargs=dict(_DEBUG)),
}


def parallelize_hf(model: nn.Module, *, parallel_dims: Any, training: Any, parallelism: Any, ac_config: Any,
                   **_: Any) -> nn.Module:
    from torch.distributed.algorithms._checkpoint.checkpoint_wrapper import checkpoint_wrapper

    from torchtitan_b200.config import TORCH_DTYPE_MAP
    from torchtitan_b200.parallel.fsdp import dp_mesh

    pd = parallel_dims
    if pd.tp_enabled or pd.cp_enabled or pd.pp_enabled or pd.ep_enabled:
        raise NotImplementedError("the HF backend supports data parallelism (FSDP2/HSDP) only")
    layers = model.decoder_layers()
    if ac_config.mode != "none":
        every = 1 if ac_config.mode == "full" or ac_config.selective_ac_option == "op" \
            else int(ac_config.selective_ac_option)
        for i in range(len(layers)):
            if i % every == 0:
                layers[i] = checkpoint_wrapper(layers[i], preserve_rng_state=ac_config.preserve_rng_state)
    if pd.dp_enabled:
        from torch.distributed.fsdp import MixedPrecisionPolicy, fully_shard

        mp = MixedPrecisionPolicy(param_dtype=TORCH_DTYPE_MAP[training.mixed_precision_param],
                                  reduce_dtype=TORCH_DTYPE_MAP[training.mixed_precision_reduce])
        mesh = dp_mesh(pd)
        import torch.distributed as dist

        gloo = dist.get_backend() == "gloo"
        model._fsdp_grad_compensation = mesh.size() if gloo else 1
        for i in range(len(layers)):
            fully_shard(layers[i], mesh=mesh, mp_policy=mp)
        fsdp_root = fully_shard(model, mesh=mesh, mp_policy=mp)
        if not gloo:
            for mod in model.modules():
                if hasattr(mod, "set_gradient_divide_factor"):
                    mod.set_gradient_divide_factor(1.0)
        del fsdp_root
    return model


def model_registry(flavor: str) -> ModelSpec:
    if flavor not in hf_args:
        raise ValueError(f"unknown hf_transformers flavor '{flavor}', available: {sorted(hf_args)}")
    return ModelSpec(name="hf_transformers", flavor=flavor, model=copy.deepcopy(hf_args[flavor]),
                     parallelize_fn=parallelize_hf, pipelining_fn=None, build_loss_fn=build_cross_entropy_loss)


__all__ = ["HFCausalLM", "HFModelArgs", "model_registry", "hf_args"]
