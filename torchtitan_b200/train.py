"""Entry point: ``torchrun ... -m torchtitan_b200.train --module llama3 --config llama3_debugmodel [--sec.key v]``
(parity: ``torchtitan/train.py:16-64``)."""
from __future__ import annotations

import os

import torch

from torchtitan_b200.config.manager import ConfigManager
from torchtitan_b200.utils.logging import init_logger, logger


def main(trainer_cls=None) -> None:
    init_logger()
    cfg = ConfigManager().parse_args()
    if trainer_cls is None:  # the config names its trainer (e.g. FluxTrainer.Config)
        from torchtitan_b200.trainer import Trainer

        owner = getattr(type(cfg), "_owner", None)
        trainer_cls = owner if isinstance(owner, type) and issubclass(owner, Trainer) else Trainer
    trainer = None
    try:
        trainer = trainer_cls(cfg)
        if cfg.checkpoint.create_seed_checkpoint:
            if int(os.environ.get("WORLD_SIZE", "1")) != 1:
                raise ValueError("seed checkpoints must be created on a single device")
            if not cfg.checkpoint.enable:
                raise ValueError("enable checkpointing to create a seed checkpoint")
            trainer.checkpointer.save_seed()
            logger.info("created seed checkpoint")
        else:
            trainer.train()
    finally:
        if trainer is not None:
            trainer.close()
        if torch.distributed.is_initialized():
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
