"""Periodic validation (parity: ``torchtitan/components/validate.py:30-331``):
every ``freq`` steps run ``steps`` batches (-1 = until exhausted) of a
validation dataloader without gradients and log the token-normalised loss."""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any

import torch

from torchtitan_b200.components.dataloader import BaseDataLoader, SyntheticDataLoader
from torchtitan_b200.components.loss import IGNORE_INDEX
from torchtitan_b200.config import Configurable
from torchtitan_b200.parallel import utils as dist_utils
from torchtitan_b200.utils.logging import logger


class BaseValidator(Configurable):
    @dataclass(kw_only=True, slots=True)
    class Config(Configurable.Config):
        freq: int = 10
        enable: bool = False

    def should_validate(self, step: int) -> bool:
        return step == 1 or step % self.config.freq == 0


class Validator(BaseValidator):
    @dataclass(kw_only=True, slots=True)
    class Config(BaseValidator.Config):
        steps: int = -1
        dataloader: Any = field(default_factory=lambda: SyntheticDataLoader.Config(seed=4321))

    def __init__(self, config: Config, *, dp_world_size: int = 1, dp_rank: int = 0, tokenizer: Any = None,
                 parallel_dims: Any = None, loss_fn: Any = None, validation_context: Any = None,
                 metrics_processor: Any = None, seq_len: int = 2048, local_batch_size: int = 1,
                 pp_schedule: Any = None, pp_has_first_stage: Any = None, pp_has_last_stage: Any = None,
                 device: Any = None, **kw: Any):
        self.config = config
        self.loss_fn = loss_fn
        self.parallel_dims = parallel_dims
        self.metrics_processor = metrics_processor
        self.ctx = validation_context
        self.device = device
        self.dataloader: BaseDataLoader = config.dataloader.build(
            dp_world_size=dp_world_size, dp_rank=dp_rank, tokenizer=tokenizer, seq_len=seq_len,
            local_batch_size=local_batch_size)

    @torch.no_grad()
    def validate(self, model_parts: list, step: int) -> float:
        model = model_parts[0]
        was_training = model.training
        model.eval()
        total, ntok = 0.0, 0
        for i, (inp, labels) in enumerate(self.dataloader):
            if 0 <= self.config.steps <= i:
                break
            dev = self.device or next(model.parameters()).device
            tokens = inp["input"].to(dev)
            labels = labels.to(dev)
            pred = model(tokens)
            total += float(self.loss_fn(pred, labels))
            ntok += int((labels != IGNORE_INDEX).sum())
        if self.parallel_dims is not None and self.parallel_dims.dp_enabled:
            mesh = self.parallel_dims.get_mesh("batch")
            total = float(dist_utils.dist_sum(torch.tensor(total), mesh))
            ntok = int(dist_utils.dist_sum(torch.tensor(float(ntok)), mesh))
        loss = total / max(ntok, 1)
        logger.info(f"validate step {step}: loss {loss:.5f}")
        if self.metrics_processor is not None:
            self.metrics_processor.logger.log({"validation_metrics/loss": loss}, step)
        if was_training:
            model.train()
        return loss
