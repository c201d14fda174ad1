"""Named training configs for the Llama 3 + SigLIP2 VLM (``--module vlm --config <fn>``):
synthetic image-text batches in the padded native-patch layout."""
from __future__ import annotations

from torchtitan_b200.components.checkpoint import CheckpointManager
from torchtitan_b200.components.lr_scheduler import LRSchedulersContainer
from torchtitan_b200.components.metrics import MetricsProcessor
from torchtitan_b200.components.mm_dataloader import SyntheticImageTextDataLoader
from torchtitan_b200.components.optimizer import OptimizersContainer
from torchtitan_b200.components.tokenizer import SyntheticTokenizer
from torchtitan_b200.components.validate import Validator
from torchtitan_b200.config import ActivationCheckpointConfig, ParallelismConfig, TrainingConfig
from torchtitan_b200.trainer import Trainer

from . import model_registry


def _base(flavor: str, lr: float, lbs: int, seq: int, images: int, image_size: int) -> Trainer.Config:
    spec = model_registry(flavor)
    a = spec.model
    return Trainer.Config(
        model_spec=spec,
        tokenizer=SyntheticTokenizer.Config(vocab_size=a.vocab_size),
        dataloader=SyntheticImageTextDataLoader.Config(images_per_sample=images, image_size=image_size,
                                                       patch_size=a.patch_size, vision_token_id=a.image_token_id,
                                                       layout="padded"),
        optimizer=OptimizersContainer.Config(lr=lr),
        lr_scheduler=LRSchedulersContainer.Config(warmup_steps=2, decay_ratio=0.8, decay_type="linear",
                                                  min_lr_factor=0.0),
        training=TrainingConfig(local_batch_size=lbs, seq_len=seq, steps=10),
        metrics=MetricsProcessor.Config(log_freq=1),
        parallelism=ParallelismConfig(enable_sequence_parallel=False),
        checkpoint=CheckpointManager.Config(interval=500),
        activation_checkpoint=ActivationCheckpointConfig(mode="selective"),
        validator=Validator.Config(freq=500, steps=10),
    )


def vlm_debugmodel() -> Trainer.Config:
    return _base("debugmodel", 8e-4, 8, 2048, 2, 128)


def vlm_8b_so400m() -> Trainer.Config:
    c = _base("8B_so400m", 2e-5, 1, 8192, 4, 512)
    c.training.steps = 1000
    return c
