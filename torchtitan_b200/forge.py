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
token normalisation, gradient clipping, optimizer and scheduler step.  Every
entry point works under every parallelism the trainer builds, pipeline
parallelism included:

* ``train_on_batches(batches, loss_fn=f, count_valid=c)`` swaps the summed
  per-microbatch objective ``f(pred, labels)`` (and the count it is normalised by)
  for one step.  Under pipeline parallelism the last stage evaluates ``f`` inside
  the schedule, so any objective of the model's output and a per-token target
  tensor (e.g. token ids with advantages in a second channel) trains through the
  pipeline.
* ``step_with_loss(loss_fn)`` takes an objective of the whole model (no pipeline).
* ``forward`` runs the model without gradients; under pipeline parallelism the
  stages hand activations to each other with point-to-point sends in stage order
  and the last stage's output is broadcast to every pipeline rank.

The reference's engine (``experiments/forge/engine.py:93-281``) builds the same
state and leaves the step to its caller (``experiments/forge/example_train.py``);
here the step functions are part of the engine.
"""
from __future__ import annotations

from contextlib import contextmanager
from typing import Any, Callable

import torch
import torch.distributed as dist

from torchtitan_b200.trainer import Trainer

# header layout for activations handed between pipeline stages: [ndim, dtype code, dims...]
_MAX_DIMS = 6
_DTYPES = [torch.float32, torch.bfloat16, torch.float16, torch.int64, torch.int32, torch.float64]


class ForgeEngine:
    def __init__(self, config: Trainer.Config):
        self.trainer = Trainer(config)
        self._stage_owner: list[int] | None = None

    @property
    def model_parts(self):
        return self.trainer.model_parts

    @property
    def step(self) -> int:
        return self.trainer.step

    @contextmanager
    def _objective(self, loss_fn: Callable | None, count_valid: Callable | None):
        t = self.trainer
        saved = (t.loss_fn, t.__dict__.get("count_valid"))
        if loss_fn is not None:
            t.loss_fn = loss_fn
        if count_valid is not None:
            t.count_valid = count_valid
        try:
            yield
        finally:
            t.loss_fn = saved[0]
            if saved[1] is None:
                t.__dict__.pop("count_valid", None)
            else:
                t.count_valid = saved[1]

    def train_on_batches(self, batches: list[tuple[dict[str, torch.Tensor], torch.Tensor]],
                         loss_fn: Callable[[torch.Tensor, torch.Tensor], torch.Tensor] | None = None,
                         count_valid: Callable[[torch.Tensor], torch.Tensor] | None = None) -> torch.Tensor:
        """One optimizer step over ``batches``.  ``loss_fn(pred, labels)`` returns the SUM of
        the microbatch's per-token objective (default: the model's cross entropy);
        ``count_valid(labels)`` the number of tokens it sums over (default: labels that are not
        the ignore index).  The step minimises the global sum divided by the global count."""
        t = self.trainer
        if len(batches) != t.gradient_accumulation_steps:
            raise ValueError(f"expected {t.gradient_accumulation_steps} microbatches, got {len(batches)}")
        t.step += 1
        with self._objective(loss_fn, count_valid):
            return t.train_step(iter(batches))

    def step_with_loss(self, loss_fn) -> torch.Tensor:
        """One optimizer step on ``loss_fn(model)``, any differentiable per-rank objective
        (e.g. an RL surrogate).  The step minimises the mean of the ranks' objectives over
        the data-parallel ranks, with the trainer's gradient finish, clipping, optimizer and
        LR step.  Returns this rank's objective.  Under pipeline parallelism no rank holds
        the whole model: use ``train_on_batches`` with a ``loss_fn`` of the last stage's output."""
        t = self.trainer
        pd = t.parallel_dims
        if pd.pp_enabled:
            raise ValueError("step_with_loss needs the whole model on each rank; under pipeline "
                             "parallelism pass loss_fn(pred, labels) to train_on_batches")
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

    # ------------------------------------------------------------------ forward only
    @torch.no_grad()
    def forward(self, input_dict: dict[str, torch.Tensor]) -> torch.Tensor:
        t = self.trainer
        tokens = input_dict["input"].to(t.device)
        parts = t.model_parts
        was = [m.training for m in parts]
        for m in parts:
            m.eval()
        try:
            if t.parallel_dims.pp_enabled:
                return self._pp_forward(tokens)
            return parts[0](tokens)
        finally:
            for m, w in zip(parts, was):
                m.train(w)

    def _pp_stages(self) -> list:
        sched = self.trainer.pp_schedule
        stages = getattr(sched, "_stages", None)
        return list(stages) if stages is not None else [sched._stage]

    def _pp_forward(self, tokens: torch.Tensor) -> torch.Tensor:
        """Stage-ordered forward through the pipeline: each stage's owner receives the previous
        stage's activation (point-to-point over the pipeline group), runs its part and sends
        the result on; the last stage's output goes to every pipeline rank."""
        t = self.trainer
        pp_mesh = t.parallel_dims.get_mesh("pp")
        group = pp_mesh.get_group()
        me = pp_mesh.get_local_rank()
        stages = {s.stage_index: s for s in self._pp_stages()}
        if self._stage_owner is None:
            owned = [None] * pp_mesh.size()
            dist.all_gather_object(owned, sorted(stages), group=group)
            owner = {sid: r for r, sids in enumerate(owned) for sid in sids}
            self._stage_owner = [owner[i] for i in range(len(owner))]
        owner = self._stage_owner
        n = len(owner)
        # gloo moves CPU tensors; NCCL device tensors
        comm_dev = torch.device("cpu") if dist.get_backend(group) == "gloo" else t.device
        g = lambda r: dist.get_global_rank(group, r)  # noqa: E731
        x = None
        for sid in range(n):
            if owner[sid] != me:
                continue
            if sid == 0:
                x = tokens
            elif owner[sid - 1] != me:
                x = _recv_tensor(g(owner[sid - 1]), group, comm_dev).to(t.device)
            x = stages[sid].submod(x)
            if sid + 1 < n and owner[sid + 1] != me:
                _send_tensor(x, g(owner[sid + 1]), group, comm_dev)
        last = owner[n - 1]
        if me == last:
            out = x.contiguous()
            hdr = _header(out, comm_dev)
        else:
            hdr = torch.zeros(2 + _MAX_DIMS, dtype=torch.int64, device=comm_dev)
        dist.broadcast(hdr, src=g(last), group=group)
        if me != last:
            out = torch.empty(_shape(hdr), dtype=_DTYPES[int(hdr[1])], device=comm_dev)
        buf = out.to(comm_dev)
        dist.broadcast(buf, src=g(last), group=group)
        return buf.to(t.device)

    def save(self, last_step: bool = False) -> None:
        self.trainer.checkpointer.save(self.trainer.step, last_step=last_step)

    def load(self, step: int = -1) -> bool:
        return self.trainer.checkpointer.load(step)

    def close(self) -> None:
        self.trainer.close()

    def __getattr__(self, name: str) -> Any:  # anything else of the trainer
        return getattr(self.trainer, name)


def example_train(engine: ForgeEngine, steps: int | None = None) -> list[float]:
    """A training loop written against the engine alone (parity: reference
    ``experiments/forge/example_train.py``): pulls microbatches from the configured data
    loader, steps, checkpoints and validates on the configured cadence.  Returns the losses."""
    t = engine.trainer
    c = t.config
    engine.load(c.checkpoint.load_step)
    steps = c.training.steps if steps is None else steps
    it = t.batch_generator(t.dataloader)
    losses = []
    while engine.step < steps:
        t.gc_handler.run(engine.step + 1)
        batches = [next(it) for _ in range(t.gradient_accumulation_steps)]
        losses.append(float(engine.train_on_batches(batches)))
        engine.save(last_step=engine.step == steps)
        if t.validator is not None and t.validator.should_validate(engine.step):
            t.validator.validate(t.model_parts, engine.step)
    return losses


def main(argv: list[str] | None = None) -> None:
    from torchtitan_b200.config.manager import ConfigManager

    engine = ForgeEngine(ConfigManager().parse_args(argv))
    try:
        example_train(engine)
    finally:
        engine.close()


def _header(x: torch.Tensor, dev: torch.device) -> torch.Tensor:
    if x.dim() > _MAX_DIMS or x.dtype not in _DTYPES:
        raise ValueError(f"cannot hand a {x.dtype} tensor of {x.dim()} dims between stages")
    h = [x.dim(), _DTYPES.index(x.dtype)] + list(x.shape) + [0] * (_MAX_DIMS - x.dim())
    return torch.tensor(h, dtype=torch.int64, device=dev)


def _shape(h: torch.Tensor) -> list[int]:
    return [int(v) for v in h[2:2 + int(h[0])]]


def _send_tensor(x: torch.Tensor, dst: int, group, dev: torch.device) -> None:
    if not torch.is_tensor(x):
        raise ValueError("pipeline stages must return one tensor for forward-only use")
    x = x.contiguous()
    dist.send(_header(x, dev), dst, group=group)
    dist.send(x.to(dev), dst, group=group)


def _recv_tensor(src: int, group, dev: torch.device) -> torch.Tensor:
    h = torch.empty(2 + _MAX_DIMS, dtype=torch.int64, device=dev)
    dist.recv(h, src, group=group)
    x = torch.empty(_shape(h), dtype=_DTYPES[int(h[1])], device=dev)
    dist.recv(x, src, group=group)
    return x


if __name__ == "__main__":
    main()
