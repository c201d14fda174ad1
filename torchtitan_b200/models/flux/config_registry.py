"""Named training configs for FLUX (``--module flux --config <fn>``).  The debug config
trains on synthetic image-caption pairs with random-weight text encoders and
autoencoder; the full configs expect the encoders and ``ae.safetensors`` on local disk."""
from __future__ import annotations

from torchtitan_b200.components.checkpoint import CheckpointManager
from torchtitan_b200.components.lr_scheduler import LRSchedulersContainer
from torchtitan_b200.components.metrics import MetricsProcessor
from torchtitan_b200.components.optimizer import OptimizersContainer
from torchtitan_b200.components.validate import Validator
from torchtitan_b200.config import ActivationCheckpointConfig, ParallelismConfig, TrainingConfig

from . import model_registry
from .data import FluxDataLoader
from .encoders import FluxEncoderConfig
from .trainer import FluxTrainer


def _base(flavor: str, lr: float, lbs: int, img: int, t5_len: int, steps: int, warmup: int,
          random_encoders: bool) -> FluxTrainer.Config:
    return FluxTrainer.Config(
        model_spec=model_registry(flavor),
        tokenizer=None,
        encoder=FluxEncoderConfig(max_t5_encoding_len=t5_len, random_init=random_encoders),
        dataloader=FluxDataLoader.Config(img_size=img, prompt_dropout_prob=0.447),
        optimizer=OptimizersContainer.Config(lr=lr),
        lr_scheduler=LRSchedulersContainer.Config(warmup_steps=warmup, decay_ratio=0.0),
        # seq_len: transformer tokens per sample (image patches + T5 tokens), for FLOPs and throughput
        training=TrainingConfig(local_batch_size=lbs, seq_len=(img // 16) ** 2 + t5_len, steps=steps, max_norm=2.0),
        metrics=MetricsProcessor.Config(log_freq=1 if steps <= 100 else 100),
        parallelism=ParallelismConfig(),
        checkpoint=CheckpointManager.Config(interval=1000),
        activation_checkpoint=ActivationCheckpointConfig(mode="full"),
        validator=Validator.Config(enable=False),
    )


def flux_debugmodel() -> FluxTrainer.Config:
    return _base("flux-debug", 8e-4, 4, 256, 256, 10, 1, True)


def flux_schnell() -> FluxTrainer.Config:
    return _base("flux-schnell", 1e-4, 32, 256, 256, 30000, 3000, False)


def flux_dev() -> FluxTrainer.Config:
    return _base("flux-dev", 1e-4, 32, 256, 512, 30000, 3000, False)
