"""Warmup-stable-decay LR schedule (parity: ``torchtitan/components/lr_scheduler.py:26-228``).

Factor(step): linear warmup over ``warmup_steps``; constant; then decay over
the last ``decay_ratio`` of ``total_steps`` (linear / sqrt / cosine) from 1 to
``min_lr_factor``.  One LambdaLR per optimizer; state is saved from the first
scheduler only (all schedulers are identical).
"""
from __future__ import annotations

import functools
import math
from dataclasses import dataclass
from typing import Any, Literal

from torch.distributed.checkpoint.stateful import Stateful
from torch.optim.lr_scheduler import LambdaLR

from torchtitan_b200.config import Configurable
from torchtitan_b200.utils.logging import logger


def wsd_factor(step: int, *, warmup: int, stable: int, decay: int, kind: str, min_factor: float) -> float:
    if step < warmup:
        return (step + 1) / warmup
    if step < warmup + stable:
        return 1.0
    progress = (step + 1 - warmup - stable) / max(decay, 1)
    progress = min(max(progress, 0.0), 1.0)
    if kind == "linear":
        f = 1.0 - progress
    elif kind == "sqrt":
        f = 1.0 - math.sqrt(progress)
    elif kind == "cosine":
        f = 0.5 * (1.0 + math.cos(math.pi * progress))
    else:
        raise ValueError(f"unknown decay type {kind}")
    return min_factor + (1.0 - min_factor) * f


class LRSchedulersContainer(Stateful, Configurable):
    @dataclass(kw_only=True, slots=True)
    class Config(Configurable.Config):
        warmup_steps: int = 200
        total_steps: int | None = None
        decay_ratio: float | None = None
        decay_type: Literal["linear", "sqrt", "cosine"] = "linear"
        min_lr_factor: float = 0.0

    def __init__(self, config: Config, *, optimizers: Any, training_steps: int):
        total = config.total_steps if config.total_steps is not None else training_steps
        warm = min(int(config.warmup_steps), total)
        if config.warmup_steps > total:
            logger.warning(f"warmup_steps {config.warmup_steps} > total {total}; clamped")
        decay = round(total * config.decay_ratio) if config.decay_ratio is not None else total - warm
        decay = min(decay, total - warm)
        stable = total + 1 - warm - decay
        fn = functools.partial(
            wsd_factor, warmup=warm, stable=stable, decay=decay, kind=config.decay_type, min_factor=config.min_lr_factor
        )
        self.schedulers = [LambdaLR(opt, lr_lambda=fn) for opt in optimizers]

    def __iter__(self):
        return iter(self.schedulers)

    def __len__(self) -> int:
        return len(self.schedulers)

    def step(self) -> None:
        for s in self.schedulers:
            s.step()

    def state_dict(self) -> dict[str, Any]:
        return self.schedulers[0].state_dict()

    def load_state_dict(self, sd: dict[str, Any]) -> None:
        for s in self.schedulers:
            s.load_state_dict(dict(sd))
