"""torch.profiler traces and CUDA memory snapshots on a step schedule.

Behaviour parity with ``torchtitan/tools/profiling.py:22-213``: a trace window of
``profiler_warmup + profiler_active`` steps ending on every ``profile_freq``-th
step, written per rank under ``<dump>/<save_traces_folder>/iteration_<N>``;
memory snapshots dumped every ``profile_freq`` steps and on OOM.
"""
from __future__ import annotations

import contextlib
import os
import pickle
import time
from dataclasses import dataclass

import torch

from .logging import logger

_MAX_MEM_EVENTS = 100000


@dataclass(kw_only=True, slots=True)
class ProfilingConfig:
    enable_profiling: bool = False
    save_traces_folder: str = "profile_traces"
    profile_freq: int = 10
    profiler_active: int = 1
    profiler_warmup: int = 3
    enable_memory_snapshot: bool = False
    save_memory_snapshot_folder: str = "memory_snapshot"


def _rank() -> int:
    return torch.distributed.get_rank() if torch.distributed.is_initialized() else 0


@contextlib.contextmanager
def maybe_enable_profiling(cfg: ProfilingConfig, *, global_step: int = 0, base_folder: str = ""):
    if not cfg.enable_profiling:
        yield None
        return
    trace_dir = os.path.join(base_folder, cfg.save_traces_folder)
    freq, active, warm = cfg.profile_freq, cfg.profiler_active, cfg.profiler_warmup
    if warm + active > freq:
        raise ValueError("profiler_warmup + profiler_active must not exceed profile_freq")
    wait = freq - (warm + active)

    def on_ready(prof):
        d = os.path.join(trace_dir, f"iteration_{prof.step_num}")
        os.makedirs(d, exist_ok=True)
        t0 = time.perf_counter()
        prof.export_chrome_trace(os.path.join(d, f"rank{_rank()}_trace.json"))
        logger.info(f"profiler trace written in {time.perf_counter() - t0:.2f}s to {d}")

    acts = [torch.profiler.ProfilerActivity.CPU]
    if torch.cuda.is_available():
        acts.append(torch.profiler.ProfilerActivity.CUDA)
    with torch.profiler.profile(
        activities=acts,
        schedule=torch.profiler.schedule(wait=wait, warmup=warm, active=active),
        on_trace_ready=on_ready,
        record_shapes=True,
    ) as prof:
        prof.step_num = global_step
        yield prof


class _MemorySnapshotter:
    def __init__(self, folder: str, freq: int, step: int):
        self.folder, self.freq, self.step_num = folder, freq, step
        torch.cuda.memory._record_memory_history(max_entries=_MAX_MEM_EVENTS)

    def step(self, exit_ctx: bool = False) -> None:
        self.step_num += 1
        if not exit_ctx and self.step_num % self.freq != 0:
            return
        tag = f"iteration_{self.step_num}" + ("_exit" if exit_ctx else "")
        d = os.path.join(self.folder, tag)
        os.makedirs(d, exist_ok=True)
        with open(os.path.join(d, f"rank{_rank()}_memory_snapshot.pickle"), "wb") as f:
            pickle.dump(torch.cuda.memory._snapshot(), f)


@contextlib.contextmanager
def maybe_enable_memory_snapshot(cfg: ProfilingConfig, *, global_step: int = 0, base_folder: str = ""):
    if not (cfg.enable_memory_snapshot and torch.cuda.is_available()):
        yield None
        return
    snap = _MemorySnapshotter(os.path.join(base_folder, cfg.save_memory_snapshot_folder), cfg.profile_freq, global_step)
    try:
        yield snap
    except torch.OutOfMemoryError:
        snap.step(exit_ctx=True)
        raise
