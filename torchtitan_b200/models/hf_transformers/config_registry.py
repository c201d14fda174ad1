"""Named training configs for HF-backend models (``--module hf_transformers``)."""
from __future__ import annotations

from torchtitan_b200.models.qwen3.config_registry import _base
from torchtitan_b200.trainer import Trainer

from . import model_registry


def hf_transformers_llama_debugmodel() -> Trainer.Config:
    c = _base("debugmodel", 2048, 8e-4, 8, 512)
    c.model_spec = model_registry("llama_debugmodel")
    return c


def hf_transformers_qwen3_debugmodel() -> Trainer.Config:
    c = _base("debugmodel", 2048, 8e-4, 8, 512)
    c.model_spec = model_registry("qwen3_debugmodel")
    return c
