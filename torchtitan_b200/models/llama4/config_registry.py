"""Named training configs for Llama 4 (``--module llama4 --config <fn>``)."""
from __future__ import annotations

from torchtitan_b200.config import ActivationCheckpointConfig, ParallelismConfig
from torchtitan_b200.models.qwen3.config_registry import _base as _qwen_base
from torchtitan_b200.trainer import Trainer

from . import model_registry


def _base(flavor: str, vocab: int, lr: float, lbs: int, seq: int) -> Trainer.Config:
    c = _qwen_base("debugmodel", vocab, lr, lbs, seq)
    c.model_spec = model_registry(flavor)
    return c


def llama4_debugmodel() -> Trainer.Config:
    return _base("debugmodel", 2048, 8e-4, 8, 2048)


def llama4_17bx16e() -> Trainer.Config:
    c = _base("17bx16e", 202048, 4e-3, 8, 8192)
    c.training.steps = 3000
    c.parallelism = ParallelismConfig(tensor_parallel_degree=8, expert_parallel_degree=1)
    c.activation_checkpoint = ActivationCheckpointConfig(mode="full")
    return c


def llama4_17bx128e() -> Trainer.Config:
    c = llama4_17bx16e()
    c.model_spec = model_registry("17bx128e")
    c.parallelism = ParallelismConfig(pipeline_parallel_degree=4, expert_parallel_degree=8)
    return c
