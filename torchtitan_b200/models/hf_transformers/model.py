"""Train any Hugging Face ``transformers`` causal LM with this framework's trainer
(behaviour parity: reference ``experiments/transformers_modeling_backend/model.py:83``).

The HF model is built from its config (``AutoModelForCausalLM.from_config``) on
the meta device like every other family, initialised with HF's own init, and
parallelized generically: FSDP2 on every decoder layer (the first
``nn.ModuleList`` under the model), the embeddings and the head; activation
checkpointing on the same layers.  Its compute runs HF's PyTorch modules, not
this framework's kernels -- the point of the backend is coverage.
"""
from __future__ import annotations

import dataclasses
from typing import Any

import torch
import torch.nn as nn

from torchtitan_b200.protocols import BaseModel, BaseModelArgs


@dataclasses.dataclass(kw_only=True)
class HFModelArgs(BaseModelArgs):
    model_type: str = "llama"
    config_kwargs: dict = dataclasses.field(default_factory=dict)

    @property
    def vocab_size(self) -> int:
        return int(self.config_kwargs.get("vocab_size", 32000))

    def hf_config(self):
        from transformers import AutoConfig

        return AutoConfig.for_model(self.model_type, **self.config_kwargs)

    def update_from_config(self, trainer_config: Any) -> None:
        seq = trainer_config.training.seq_len
        if self.config_kwargs.get("max_position_embeddings", 0) < seq:
            self.config_kwargs["max_position_embeddings"] = seq

    def build(self) -> "HFCausalLM":
        return HFCausalLM(self)

    def get_nparams_and_flops(self, model: nn.Module, seq_len: int) -> tuple[int, float]:
        c = model.hf.config
        nparams = sum(p.numel() for p in model.parameters())
        emb = model.hf.get_input_embeddings().weight.numel()
        head_dim = getattr(c, "head_dim", None) or c.hidden_size // c.num_attention_heads
        flops = 6 * (nparams - emb) + 6 * c.num_hidden_layers * c.num_attention_heads * 2 * head_dim * seq_len
        return nparams, float(flops)


class HFCausalLM(BaseModel):
    def __init__(self, a: HFModelArgs):
        super().__init__()
        from transformers import AutoModelForCausalLM

        self.model_args = a
        cfg = a.hf_config()
        cfg.use_cache = False
        self.hf = AutoModelForCausalLM.from_config(cfg)

    def decoder_layers(self) -> nn.ModuleList:
        for m in self.hf.modules():
            if isinstance(m, nn.ModuleList) and len(m) == self.hf.config.num_hidden_layers:
                return m
        raise RuntimeError("could not find the decoder layer list of the HF model")

    @torch.no_grad()
    def init_weights(self, buffer_device: torch.device | None = None) -> None:
        self.hf.apply(self.hf._init_weights)
        for mod in self.hf.modules():  # rotary tables: non-persistent buffers lost on the meta device
            if hasattr(mod, "inv_freq") and hasattr(mod, "rope_type"):
                from transformers.modeling_rope_utils import ROPE_INIT_FUNCTIONS

                fn = mod.compute_default_rope_parameters if mod.rope_type == "default" else \
                    ROPE_INIT_FUNCTIONS[mod.rope_type]
                dev = buffer_device or mod.inv_freq.device
                inv, scaling = fn(mod.config, dev)
                mod.inv_freq = inv.to(dev)
                mod.original_inv_freq = inv.clone().to(dev)
                mod.attention_scaling = scaling

    def forward(self, tokens: torch.Tensor, attention_masks=None, positions=None, **kw) -> torch.Tensor:
        return self.hf(input_ids=tokens, position_ids=positions, use_cache=False).logits
