"""Named training configs for GPT-OSS (``--module gpt_oss --config <fn>``)."""
from __future__ import annotations

from torchtitan_b200.config import ActivationCheckpointConfig
from torchtitan_b200.models.qwen3.config_registry import _base as _qwen_base
from torchtitan_b200.trainer import Trainer

from . import model_registry


def gpt_oss_debugmodel() -> Trainer.Config:
    c = _qwen_base("debugmodel", 2048, 8e-4, 8, 1024)
    c.model_spec = model_registry("debugmodel")
    return c


def gpt_oss_20b() -> Trainer.Config:
    c = _qwen_base("debugmodel", 201088, 3e-4, 1, 4096)
    c.model_spec = model_registry("20b")
    c.training.steps = 1000
    c.activation_checkpoint = ActivationCheckpointConfig(mode="full")
    return c


def gpt_oss_120b() -> Trainer.Config:
    c = gpt_oss_20b()
    c.model_spec = model_registry("120b")
    return c
