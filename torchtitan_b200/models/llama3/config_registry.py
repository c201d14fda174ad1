"""Named training configs for Llama 3 (``--module llama3 --config <fn>``).

Function names follow the reference (``models/llama3/config_registry.py``);
data defaults to the synthetic uniform-token loader because this framework
ships no datasets.  ``llama3_8b_b200`` / ``llama3_70b_b200`` are the
benchmark configs of this project (FSDP2 at seq 8192, SAC / full AC).
"""
from __future__ import annotations

from torchtitan_b200.components.checkpoint import CheckpointManager
from torchtitan_b200.components.dataloader import SyntheticDataLoader
from torchtitan_b200.components.lr_scheduler import LRSchedulersContainer
from torchtitan_b200.components.metrics import MetricsProcessor
from torchtitan_b200.components.optimizer import OptimizersContainer
from torchtitan_b200.components.tokenizer import SyntheticTokenizer
from torchtitan_b200.components.validate import Validator
from torchtitan_b200.config import ActivationCheckpointConfig, ParallelismConfig, TrainingConfig
from torchtitan_b200.protocols.model_converter import ModelConvertersContainer
from torchtitan_b200.trainer import Trainer

from . import model_registry


def llama3_debugmodel() -> Trainer.Config:
    return Trainer.Config(
        model_spec=model_registry("debugmodel"),
        tokenizer=SyntheticTokenizer.Config(vocab_size=2048),
        dataloader=SyntheticDataLoader.Config(),
        optimizer=OptimizersContainer.Config(lr=8e-4),
        lr_scheduler=LRSchedulersContainer.Config(warmup_steps=2, decay_ratio=0.8, decay_type="linear",
                                                  min_lr_factor=0.0),
        training=TrainingConfig(local_batch_size=8, seq_len=2048, steps=10),
        metrics=MetricsProcessor.Config(log_freq=1),
        parallelism=ParallelismConfig(pipeline_parallel_schedule="Interleaved1F1B"),
        checkpoint=CheckpointManager.Config(interval=10, last_save_model_only=False),
        activation_checkpoint=ActivationCheckpointConfig(mode="selective"),
        validator=Validator.Config(freq=5, steps=10),
    )


def llama3_debugmodel_cpu() -> Trainer.Config:
    """Config 1 of the benchmark spec: CPU/gloo, FSDP2, fp32, seq 512, lbs 4, AdamW 8e-4, 10 steps."""
    c = llama3_debugmodel()
    c.training = TrainingConfig(local_batch_size=4, seq_len=512, steps=10, dtype="float32",
                                mixed_precision_param="float32")
    c.activation_checkpoint = ActivationCheckpointConfig(mode="none")
    return c


def llama3_debugmodel_flex_attn() -> Trainer.Config:
    c = llama3_debugmodel()
    c.model_spec = model_registry("debugmodel_flex_attn")
    return c


def llama3_debugmodel_varlen_attn() -> Trainer.Config:
    c = llama3_debugmodel()
    c.model_spec = model_registry("debugmodel_varlen_attn")
    return c


def llama3_8b() -> Trainer.Config:
    return Trainer.Config(
        model_spec=model_registry("8B"),
        tokenizer=SyntheticTokenizer.Config(vocab_size=128256),
        dataloader=SyntheticDataLoader.Config(),
        metrics=MetricsProcessor.Config(log_freq=10, enable_tensorboard=False),
        optimizer=OptimizersContainer.Config(lr=3e-4),
        training=TrainingConfig(local_batch_size=1, seq_len=8192, steps=1000),
        checkpoint=CheckpointManager.Config(interval=500),
        activation_checkpoint=ActivationCheckpointConfig(mode="selective"),
        validator=Validator.Config(freq=500, steps=1200),
    )


def llama3_70b() -> Trainer.Config:
    c = llama3_8b()
    c.model_spec = model_registry("70B")
    c.optimizer = OptimizersContainer.Config(lr=1.5e-4)
    c.training = TrainingConfig(local_batch_size=8, seq_len=8192, steps=1000)
    c.parallelism = ParallelismConfig(tensor_parallel_degree=8)
    c.activation_checkpoint = ActivationCheckpointConfig(mode="full")
    return c


def llama3_70b_fsdp2_tp4() -> Trainer.Config:
    """Config 3 of the benchmark spec: FSDP2=2 x async TP=4, full AC, seq 8192, lbs 1."""
    c = llama3_70b()
    c.training = TrainingConfig(local_batch_size=1, seq_len=8192, steps=1000)
    c.parallelism = ParallelismConfig(tensor_parallel_degree=4, enable_async_tensor_parallel=True)
    c.model_converters = ModelConvertersContainer.Config(names=["mxfp8"])
    return c


def llama3_405b() -> Trainer.Config:
    c = llama3_8b()
    c.model_spec = model_registry("405B")
    c.optimizer = OptimizersContainer.Config(lr=8e-5)
    c.lr_scheduler = LRSchedulersContainer.Config(warmup_steps=600)
    c.training = TrainingConfig(local_batch_size=2, seq_len=8192, steps=3000)
    c.parallelism = ParallelismConfig(tensor_parallel_degree=8, pipeline_parallel_degree=8,
                                      pipeline_parallel_schedule="Interleaved1F1B")
    c.activation_checkpoint = ActivationCheckpointConfig(mode="full")
    return c
