"""Reference arm of bench.py: the UNMODIFIED reference trainer (installed under
baseline/_ref) on the same metric and config as bench.py's own arm.

It goes through the reference's public API only: its ``llama3_8b`` config
function, ``Trainer.Config.build()``, ``Trainer.train_step`` and its
``batch_generator``.  The only plug-in is a synthetic-token dataloader,
written against the reference's own ``BaseDataLoader`` Configurable interface
(there is no dataset on the box).  torch.compile is enabled as in the
reference's published B200 run (per-op SAC, FSDP2); set ``TTB_REF_COMPILE=0``
to run it eagerly.  Timing, clocks and the JSON line follow bench.py exactly.
"""
from __future__ import annotations

import json
import os
import socket
import time
from dataclasses import dataclass

import torch


def _single_process_env() -> None:
    # the reference reads LOCAL_RANK etc. unconditionally; without torchrun, run as rank 0 of 1
    os.environ.setdefault("RANK", "0")
    os.environ.setdefault("LOCAL_RANK", "0")
    os.environ.setdefault("WORLD_SIZE", "1")
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    if "MASTER_PORT" not in os.environ:
        s = socket.socket()
        s.bind(("127.0.0.1", 0))
        os.environ["MASTER_PORT"] = str(s.getsockname()[1])
        s.close()


def synthetic_loader_config(vocab_size: int = 128256, seed: int = 1234):
    """Config of a synthetic-token dataloader written against the reference's own
    ``BaseDataLoader`` Configurable interface (there is no dataset on the box): uniform
    tokens from a seeded generator per (rank, batch), pinned, yielded as
    ``({"input": tokens[:, :-1]}, tokens[:, 1:])``."""
    from torchtitan.components.dataloader import BaseDataLoader

    class SyntheticTokens(BaseDataLoader):
        @dataclass(kw_only=True, slots=True)
        class Config(BaseDataLoader.Config):
            vocab_size: int = 128256
            seed: int = 1234

        def __init__(self, config, *, dp_world_size=1, dp_rank=0, tokenizer=None, seq_len=8192,
                     local_batch_size=1, **kw):
            self.config, self.rank, self.seq, self.bs = config, dp_rank, seq_len, local_batch_size
            self.i = 0

        def __iter__(self):
            while True:
                g = torch.Generator().manual_seed(self.config.seed * 1_000_003 + self.rank * 7919 + self.i)
                t = torch.randint(0, self.config.vocab_size, (self.bs, self.seq + 1), generator=g)
                if torch.cuda.is_available():
                    t = t.pin_memory()
                self.i += 1
                yield {"input": t[:, :-1]}, t[:, 1:]

        def state_dict(self):
            return {"i": self.i}

        def load_state_dict(self, sd):
            self.i = sd.get("i", 0)

    return SyntheticTokens.Config(vocab_size=vocab_size, seed=seed)


def run(a, dist_env, max_over_ranks, ClockSampler, METRIC, BASELINE_TPS_PER_GPU):
    _single_process_env()
    import torch.distributed as dist
    from torchtitan.components.checkpoint import CheckpointManager
    from torchtitan.components.metrics import MetricsProcessor
    from torchtitan.distributed import utils as dist_utils
    from torchtitan.config import ActivationCheckpointConfig, CompileConfig, TrainingConfig
    from torchtitan.models.llama3 import config_registry as reg
    from torchtitan.models.llama3 import model_registry
    from torchtitan.tools.logging import init_logger
    from torchtitan.tools.profiling import ProfilingConfig

    init_logger()
    rank, world, local = dist_env()
    here = os.path.dirname(os.path.abspath(__file__))
    cfg = reg.llama3_8b()
    cfg.model_spec = model_registry(a.flavor)
    cfg.hf_assets_path = os.path.join(here, "_ref", "assets", "tokenizer")
    cfg.profiling = ProfilingConfig(enable_profiling=False)
    cfg.metrics = MetricsProcessor.Config(log_freq=10 ** 9, enable_tensorboard=False)
    cfg.training = TrainingConfig(local_batch_size=1, seq_len=a.seq_len, steps=a.warmup + 2 * a.steps + 2)
    cfg.dataloader = synthetic_loader_config()
    cfg.checkpoint = CheckpointManager.Config(enable=False)
    cfg.activation_checkpoint = ActivationCheckpointConfig(mode=a.ac)
    cfg.validator.enable = False
    use_compile = os.environ.get("TTB_REF_COMPILE", "1") == "1"
    cfg.compile = CompileConfig(enable=use_compile, components=["model", "loss"])
    cfg.dump_folder = os.path.join(os.environ.get("TMPDIR", "/tmp"), "ttb_ref_outputs")
    trainer = cfg.build()
    it = trainer.batch_generator(trainer.dataloader)
    tokens_per_step = a.seq_len * world

    def step():
        trainer.step += 1
        trainer.train_step(it)

    for _ in range(a.warmup):
        step()
    torch.cuda.synchronize()
    if dist.is_initialized():
        dist.barrier()
    clocks = ClockSampler(local)
    clocks.start()
    torch.cuda.synchronize()
    if dist.is_initialized():
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    if dist.is_initialized():
        dist.barrier()
    torch.cuda.synchronize()
    dev_s = max_over_ranks(e0.elapsed_time(e1) / 1e3)
    clk = clocks.stop()
    # end to end: the same sequence as the reference's ``Trainer.train_step`` (zero grad,
    # inputs copied from pinned host memory, forward/backward, clip, optimizer and LR step)
    # through its public methods, with the loss read back each step
    if dist.is_initialized():
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(a.steps):
        trainer.step += 1
        trainer.optimizers.zero_grad()
        inp, labels = next(it)
        inp = {k: v.to(trainer.device) for k, v in inp.items()}
        labels = labels.to(trainer.device)
        n = torch.tensor(float(labels.numel()), device=trainer.device) * world
        loss = trainer.forward_backward_step(input_dict=inp, labels=labels, global_valid_tokens=n)
        dist_utils.clip_grad_norm_([p for m in trainer.model_parts for p in m.parameters()],
                                   trainer.config.training.max_norm, foreach=True)
        trainer.optimizers.step()
        trainer.lr_schedulers.step()
        _ = float(loss.item())
    torch.cuda.synchronize()
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    value = tokens_per_step * a.steps / dev_s
    out = {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": round(1e3 * dev_s / a.steps, 2), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": round(value / (BASELINE_TPS_PER_GPU * world), 4), "dtype": "bf16",
        "data": "synthetic uniform tokens, random-init weights",
        "config": {"model": f"llama3_{a.flavor}", "global_batch": world, "seq_len": a.seq_len,
                   "parallelism": f"fsdp{world}", "ac": a.ac, "compile": use_compile,
                   "l2": "inputs larger than L2 (no flush)"},
        "tokens_per_sec_per_gpu": round(value / world, 1),
        "peak_mem_gib": round(torch.cuda.max_memory_reserved() / 1024 ** 3, 2),
        "clocks": clk,
        "e2e": {"value": round(tokens_per_step * a.steps / e2e_s, 1), "unit": "tokens/s",
                "h2d_bytes_per_step": a.seq_len * 8 * 2, "d2h_bytes_per_step": 4},
        "impl": "reference",
    }
    if rank == 0:
        print(json.dumps(out), flush=True)
    trainer.close()
    if dist.is_initialized():
        dist.destroy_process_group()
