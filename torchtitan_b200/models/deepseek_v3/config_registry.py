"""Named training configs for DeepSeek-V3 (``--module deepseek_v3 --config <fn>``)."""
from __future__ import annotations

from torchtitan_b200.config import ActivationCheckpointConfig, ParallelismConfig
from torchtitan_b200.models.qwen3.config_registry import _base as _qwen_base
from torchtitan_b200.trainer import Trainer

from . import model_registry


def _base(flavor: str, vocab: int, lr: float, lbs: int, seq: int) -> Trainer.Config:
    c = _qwen_base("debugmodel", vocab, lr, lbs, seq)
    c.model_spec = model_registry(flavor)
    return c


def deepseek_v3_debugmodel() -> Trainer.Config:
    return _base("debugmodel", 2048, 8e-4, 8, 2048)


def deepseek_v3_debugmodel_qlora() -> Trainer.Config:
    return _base("debugmodel_qlora", 2048, 8e-4, 8, 2048)


def deepseek_v3_16b() -> Trainer.Config:
    c = _base("16B", 102400, 2.2e-4, 4, 4096)
    c.training.steps = 1000
    c.parallelism = ParallelismConfig(expert_parallel_degree=8)
    return c


def deepseek_v3_671b() -> Trainer.Config:
    c = _base("671B", 129280, 2.2e-4, 1, 4096)
    c.training.steps = 1000
    c.parallelism = ParallelismConfig(expert_parallel_degree=32, pipeline_parallel_degree=8,
                                      pipeline_parallel_schedule="Interleaved1F1B")
    c.activation_checkpoint = ActivationCheckpointConfig(mode="full")
    return c
