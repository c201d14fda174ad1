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

    loss_step = None
    """Set by the trainer: ``loss_step(input_dict, labels) -> loss sum`` of this rank's share of
    the batch through the training layout (pipeline ``eval`` schedule, context-parallel
    sharding, vocabulary-parallel loss); 0 on pipeline stages without the loss."""

    @torch.no_grad()
    def validate(self, model_parts: list, step: int) -> float:
        import torch.distributed as dist

        was_training = [m.training for m in model_parts]
        for m in model_parts:
            m.eval()
        model = model_parts[0]
        dev = self.device or next(model.parameters()).device
        total = torch.zeros((), dtype=torch.float64)
        ntok = 0
        for i, (inp, labels) in enumerate(self.dataloader):
            if 0 <= self.config.steps <= i:
                break
            inp = {k: (v.to(dev) if torch.is_tensor(v) else v) for k, v in inp.items()}
            labels = labels.to(dev)
            if self.loss_step is not None:
                total += float(self.loss_step(inp, labels))
            else:
                total += float(self.loss_fn(model(inp["input"]), labels))
            ntok += int((labels != IGNORE_INDEX).sum())
        pd = self.parallel_dims
        if pd is not None and pd.pp_enabled:  # only the last stage holds the loss
            pp = pd.get_mesh("pp")
            t = total.reshape(1).to(dev if dist.get_backend() != "gloo" else "cpu")
            dist.broadcast(t, src=dist.get_global_rank(pp.get_group(), pp.size() - 1), group=pp.get_group())
            total = t.reshape(()).cpu()
        if pd is not None and pd.dp_cp_enabled:
            total = dist_utils.dist_sum(total.float(), pd.get_mesh("loss"))  # dp and cp shards
        if pd is not None and pd.dp_enabled:
            ntok = int(dist_utils.dist_sum(torch.tensor(float(ntok)), pd.get_mesh("batch")))
        loss = float(total) / max(ntok, 1)
        logger.info(f"validate step {step}: loss {loss:.5f}")
        if self.metrics_processor is not None:
            self.metrics_processor.logger.log({"validation_metrics/loss": loss}, step)
        for m, w in zip(model_parts, was_training):
            m.train(w)
        return loss
