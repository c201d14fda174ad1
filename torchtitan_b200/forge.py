"""Post-training engine (parity: reference ``experiments/forge/engine.py:35``): the
trainer's construction -- meshes, parallelized model, optimizer, LR schedule,
checkpointing -- without its data loader loop, for callers (RL, SFT drivers)
that produce their own batches.

    engine = ForgeEngine(config)
    loss = engine.train_on_batches([({"input": tokens}, labels), ...])   # one optimizer step
    logits = engine.forward({"input": tokens})                           # no grad
    engine.save()

``train_on_batches`` takes exactly ``gradient_accumulation_steps`` microbatches
(one by default) and runs the same step as ``Trainer.train_step``: global
token normalisation, gradient clipping, optimizer and scheduler step.
"""
from __future__ import annotations

from typing import Any

import torch

from torchtitan_b200.trainer import Trainer


class ForgeEngine:
    def __init__(self, config: Trainer.Config):
        self.trainer = Trainer(config)

    @property
    def model_parts(self):
        return self.trainer.model_parts

    @property
    def step(self) -> int:
        return self.trainer.step

    def train_on_batches(self, batches: list[tuple[dict[str, torch.Tensor], torch.Tensor]]) -> torch.Tensor:
        t = self.trainer
        if len(batches) != t.gradient_accumulation_steps:
            raise ValueError(f"expected {t.gradient_accumulation_steps} microbatches, got {len(batches)}")
        t.step += 1
        return t.train_step(iter(batches))

    def step_with_loss(self, loss_fn) -> torch.Tensor:
        """One optimizer step on ``loss_fn(model)``, any differentiable per-rank objective
        (e.g. an RL surrogate).  The step minimises the mean of the ranks' objectives over
        the data-parallel ranks, with the trainer's gradient finish, clipping, optimizer and
        LR step.  Returns this rank's objective."""
        t = self.trainer
        pd = t.parallel_dims
        if pd.pp_enabled:
            raise NotImplementedError("custom objectives under pipeline parallelism are not wired")
        t.optimizers.zero_grad()
        model = t.model_parts[0]
        dp_rt = getattr(model, "_dp_runtime", None)
        if dp_rt is not None:
            dp_rt.begin_microbatch(0, 1)
        # data-parallel gradients are summed (not averaged) over the batch ranks
        n_dp = pd.get_mesh("batch").size() if pd.dp_enabled else 1
        comp = getattr(model, "_fsdp_grad_compensation", 1)
        t.step += 1
        with t.train_context():
            loss = loss_fn(model)
            (loss * (comp / n_dp)).backward()
        t.apply_gradients()
        return loss.detach()

    @torch.no_grad()
    def forward(self, input_dict: dict[str, torch.Tensor]) -> torch.Tensor:
        t = self.trainer
        if t.parallel_dims.pp_enabled:
            raise NotImplementedError("forward-only under pipeline parallelism is not wired")
        model = t.model_parts[0]
        was = model.training
        model.eval()
        try:
            return model(input_dict["input"].to(t.device))
        finally:
            model.train(was)

    def save(self, last_step: bool = False) -> None:
        self.trainer.checkpointer.save(self.trainer.step, last_step=last_step)

    def load(self, step: int = -1) -> bool:
        return self.trainer.checkpointer.load(step)

    def close(self) -> None:
        self.trainer.close()

    def __getattr__(self, name: str) -> Any:  # anything else of the trainer
        return getattr(self.trainer, name)
