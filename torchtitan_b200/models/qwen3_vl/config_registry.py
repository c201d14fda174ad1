"""Named training configs for Qwen3-VL (``--module qwen3_vl --config <fn>``): synthetic
image-text batches (random tokens, random images in the native-patch layout)."""
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
        dataloader=SyntheticImageTextDataLoader.Config(
            images_per_sample=images, image_size=image_size, patch_size=a.patch_size,
            temporal_patch_size=a.temporal_patch_size, merge_size=a.spatial_merge_size,
            vision_token_id=a.image_token_id),
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


def qwen3_vl_debugmodel() -> Trainer.Config:
    return _base("debugmodel", 8e-4, 8, 2048, 2, 256)


def qwen3_vl_debugmodel_moe() -> Trainer.Config:
    return _base("debugmodel_moe", 8e-4, 8, 2048, 2, 256)


def qwen3_vl_2b() -> Trainer.Config:
    c = _base("2B", 2e-5, 2, 8192, 4, 512)
    c.training.steps = 1000
    return c


def qwen3_vl_8b() -> Trainer.Config:
    c = _base("8B", 2e-5, 1, 8192, 4, 512)
    c.training.steps = 1000
    return c


def qwen3_vl_30b_a3b() -> Trainer.Config:
    c = _base("30B-A3B", 2e-5, 1, 8192, 4, 512)
    c.training.steps = 1000
    c.parallelism.expert_parallel_degree = 8
    return c


def qwen3_vl_debugmodel_cc12m() -> Trainer.Config:
    """Debug model on CC12M-format WebDataset shards (``--dataloader.dataset-path <dir of .tar>``;
    ``--dataloader.dataset obelics`` reads OBELICS parquet/JSONL instead)."""
    from torchtitan_b200.components.mm_datasets import MMDataLoader

    c = qwen3_vl_debugmodel()
    a = c.model_spec.model
    c.training.local_batch_size, c.training.seq_len = 2, 1024
    c.dataloader = MMDataLoader.Config(dataset="cc12m", dataset_path="./data/cc12m", patch_size=a.patch_size,
                                       temporal_patch_size=a.temporal_patch_size,
                                       spatial_merge_size=a.spatial_merge_size, min_pixels=64 * 64,
                                       max_pixels=256 * 256, packing_buffer_size=16,
                                       image_token_id=a.image_token_id, video_token_id=a.video_token_id,
                                       vision_start_id=a.vocab_size - 8, vision_end_id=a.vocab_size - 7)
    return c
