"""Named training configs for Kimi-Linear (``--module kimi_linear --config <fn>``).

Function names follow the reference (``kimi_linear/config_registry.py:417-896``):
``kimi_linear_<size>_{baseline,block_attn_res,full_attn_res}``.  Also the two
benchmark configs of this project:

* ``kimi_linear_48b_ep8``: 48B-A3B-style hybrid, EP=8 + FSDP2, DistMuon,
  seq 4096, local batch 2, router aux loss on.
* ``kimi_linear_48b_longctx``: seq 131072, Ulysses CP=4 x PP=2 (interleaved
  1F1B), EP=4 per stage, DistMuon, full AC.
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
from torchtitan_b200.trainer import Trainer

from . import _SWEEP, model_registry

_LR = {"194m": 2.99e-3, "241m": 2.80e-3, "296m": 2.50e-3, "436m": 2.20e-3, "528m": 2.02e-3,
       "447m_aligned": 2.20e-3, "48b": 1.0e-3}


def _base(flavor: str, lr: float = 1e-3) -> Trainer.Config:
    spec = model_registry(flavor)
    return Trainer.Config(
        model_spec=spec,
        tokenizer=SyntheticTokenizer.Config(vocab_size=spec.model.vocab_size),
        dataloader=SyntheticDataLoader.Config(),
        optimizer=OptimizersContainer.Config(lr=lr, weight_decay=0.1),
        lr_scheduler=LRSchedulersContainer.Config(warmup_steps=200, decay_ratio=0.2, decay_type="cosine"),
        training=TrainingConfig(local_batch_size=4, seq_len=2048, steps=10000, max_norm=1.0),
        metrics=MetricsProcessor.Config(log_freq=10),
        checkpoint=CheckpointManager.Config(interval=1000),
        activation_checkpoint=ActivationCheckpointConfig(mode="full"),
        validator=Validator.Config(freq=1000, steps=50),
    )


def kimi_linear_debugmodel() -> Trainer.Config:
    c = _base("debugmodel", 1e-3)
    c.training = TrainingConfig(local_batch_size=2, seq_len=128, steps=10)
    c.metrics = MetricsProcessor.Config(log_freq=1)
    c.activation_checkpoint = ActivationCheckpointConfig(mode="none")
    c.lr_scheduler = LRSchedulersContainer.Config(warmup_steps=2)
    return c


def kimi_linear_debugmodel_block_attn_res() -> Trainer.Config:
    c = kimi_linear_debugmodel()
    c.model_spec = model_registry("debugmodel_block_attn_res")
    return c


def _make(size: str, variant: str):
    def fn() -> Trainer.Config:
        return _base(f"{size}_{variant}", _LR[size])

    fn.__name__ = f"kimi_linear_{size}_{variant}"
    fn.__doc__ = f"Kimi-Linear {size} ({variant.replace('_', ' ')})."
    return fn


for _size in _SWEEP:
    for _variant in ("baseline", "block_attn_res", "full_attn_res"):
        _f = _make(_size, _variant)
        globals()[_f.__name__] = _f


def kimi_linear_48b_ep8() -> Trainer.Config:
    c = _base("48b_baseline", 1e-3)
    c.model_spec.model.aux_loss_coeff = 1e-3
    c.optimizer = OptimizersContainer.Config(name="DistMuon", lr=1e-3, muon_lr=0.02)
    c.training = TrainingConfig(local_batch_size=2, seq_len=4096, steps=1000)
    c.parallelism = ParallelismConfig(expert_parallel_degree=8)
    c.activation_checkpoint = ActivationCheckpointConfig(mode="full")
    return c


def kimi_linear_48b_longctx() -> Trainer.Config:
    c = kimi_linear_48b_ep8()
    c.training = TrainingConfig(local_batch_size=1, seq_len=131072, steps=1000)
    c.parallelism = ParallelismConfig(context_parallel_degree=4, context_parallel_method="ulysses",
                                      pipeline_parallel_degree=2, pipeline_parallel_schedule="Interleaved1F1B",
                                      expert_parallel_degree=4)
    return c
