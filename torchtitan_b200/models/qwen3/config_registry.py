"""Named training configs for Qwen3 (``--module qwen3 --config <fn>``);
synthetic data, as every config of this framework."""
from __future__ import annotations

from torchtitan_b200.components.checkpoint import CheckpointManager
from torchtitan_b200.components.dataloader import SyntheticDataLoader
from torchtitan_b200.components.lr_scheduler import LRSchedulersContainer
from torchtitan_b200.components.metrics import MetricsProcessor
from torchtitan_b200.components.optimizer import OptimizersContainer
from torchtitan_b200.components.tokenizer import SyntheticTokenizer
from torchtitan_b200.components.validate import Validator
from torchtitan_b200.config import ActivationCheckpointConfig, ParallelismConfig, TrainingConfig
from torchtitan_b200.trainer import Trainer

from . import model_registry


def _base(flavor: str, vocab: int, lr: float, lbs: int, seq: int) -> Trainer.Config:
    return Trainer.Config(
        model_spec=model_registry(flavor),
        tokenizer=SyntheticTokenizer.Config(vocab_size=vocab),
        dataloader=SyntheticDataLoader.Config(),
        optimizer=OptimizersContainer.Config(lr=lr),
        lr_scheduler=LRSchedulersContainer.Config(warmup_steps=2, decay_ratio=0.8, decay_type="linear",
                                                  min_lr_factor=0.0),
        training=TrainingConfig(local_batch_size=lbs, seq_len=seq, steps=10),
        metrics=MetricsProcessor.Config(log_freq=1),
        parallelism=ParallelismConfig(),
        checkpoint=CheckpointManager.Config(interval=500),
        activation_checkpoint=ActivationCheckpointConfig(mode="selective"),
        validator=Validator.Config(freq=500, steps=10),
    )


def qwen3_debugmodel() -> Trainer.Config:
    return _base("debugmodel", 2048, 8e-4, 8, 2048)


def qwen3_debugmodel_moe() -> Trainer.Config:
    return _base("debugmodel_moe", 2048, 8e-4, 8, 2048)


def qwen3_0_6b() -> Trainer.Config:
    c = _base("0.6B", 151936, 3e-4, 4, 4096)
    c.training.steps = 1000
    return c


def qwen3_1_7b() -> Trainer.Config:
    c = _base("1.7B", 151936, 3e-4, 4, 4096)
    c.training.steps = 1000
    return c


def qwen3_8b() -> Trainer.Config:
    c = _base("8B", 151936, 3e-4, 1, 8192)
    c.training.steps = 1000
    return c


def qwen3_32b() -> Trainer.Config:
    c = qwen3_8b()
    c.model_spec = model_registry("32B")
    c.activation_checkpoint = ActivationCheckpointConfig(mode="full")
    return c


def qwen3_30b_a3b() -> Trainer.Config:
    c = _base("30B-A3B", 151936, 3e-4, 2, 4096)
    c.training.steps = 1000
    c.parallelism = ParallelismConfig(expert_parallel_degree=8)
    return c


def qwen3_235b_a22b() -> Trainer.Config:
    c = qwen3_30b_a3b()
    c.model_spec = model_registry("235B-A22B")
    c.activation_checkpoint = ActivationCheckpointConfig(mode="full")
    return c
