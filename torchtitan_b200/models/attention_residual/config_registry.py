"""Named training configs for dense AttnRes models (``--module attention_residual``)."""
from __future__ import annotations

from torchtitan_b200.models.llama3.config_registry import llama3_8b, llama3_debugmodel
from torchtitan_b200.trainer import Trainer

from . import model_registry


def attention_residual_debugmodel() -> Trainer.Config:
    c = llama3_debugmodel()
    c.model_spec = model_registry("debugmodel")
    return c


def attention_residual_debugmodel_full() -> Trainer.Config:
    c = llama3_debugmodel()
    c.model_spec = model_registry("debugmodel_full")
    return c


def attention_residual_8b() -> Trainer.Config:
    c = llama3_8b()
    c.model_spec = model_registry("8B")
    return c
