"""Distributed checkpointing (DCP) with resume, async save, purge and HF export.

Layout (parity: ``torchtitan/components/checkpoint.py:49-53,320-330``):
``<dump>/<folder>/step-<N>/`` holding a DCP snapshot of
``{"model": flattened FQN -> tensor, "optimizer": flattened, "lr_scheduler",
"dataloader": {"dp_rank_<r>": bytes, "world_size"}, "train_state": {step,
ntokens_seen}}``.  Features: save every ``interval`` steps and at the last
step (model-only in ``export_dtype`` if ``last_save_model_only``), async save
on a background thread (optionally staged through pinned host memory), keep
the latest ``keep_latest_k`` snapshots, ``initial_load_path`` (DCP or HF
safetensors through the model's state-dict adapter), ``exclude_from_loading``,
seed checkpoints, and HF safetensors export at the last step.
"""
from __future__ import annotations

import os
import re
import shutil
import threading
import time
from concurrent.futures import Future, ThreadPoolExecutor
from dataclasses import dataclass, field
from typing import Any, Literal

import torch
import torch.distributed as dist
import torch.distributed.checkpoint as dcp
from torch.distributed.checkpoint.api import CheckpointException
import torch.nn as nn
from torch.distributed.checkpoint.state_dict import StateDictOptions, get_model_state_dict, set_model_state_dict
from torch.distributed.checkpoint.stateful import Stateful

from torchtitan_b200.config import TORCH_DTYPE_MAP, Configurable
from torchtitan_b200.utils.logging import logger

MODEL, OPTIMIZER, LR_SCHEDULER, DATALOADER, TRAIN_STATE = "model", "optimizer", "lr_scheduler", "dataloader", "train_state"


class ModelWrapper(Stateful):
    """All model parts seen as one flat FQN state dict."""

    def __init__(self, model: nn.Module | list[nn.Module]):
        self.model = [model] if isinstance(model, nn.Module) else model

    def state_dict(self) -> dict[str, Any]:
        out: dict[str, Any] = {}
        for m in self.model:
            sd = get_model_state_dict(m)
            # single-replica mixed precision: save the fp32 masters, not the bf16 compute weights
            masters = {n.replace("_checkpoint_wrapped_module.", ""): p._master
                       for n, p in m.named_parameters() if hasattr(p, "_master")}
            out.update({k: masters.get(k, v) for k, v in sd.items()})
        return out

    def load_state_dict(self, sd: dict[str, Any]) -> None:
        for m in self.model:
            named = {n.replace("_checkpoint_wrapped_module.", ""): p for n, p in m.named_parameters()}
            with torch.no_grad():
                rest = {}
                for k, v in sd.items():
                    p = named.get(k)
                    if p is not None and hasattr(p, "_master"):
                        p._master.copy_(v)
                        p.data.copy_(p._master)
                    else:
                        rest[k] = v
            set_model_state_dict(m, rest, options=StateDictOptions(strict=False))
            rt = getattr(m, "_dp_runtime", None)
            if rt is not None:  # weights are views of the runtime's buffer; its masters follow them
                rt.masters_from_weights()


def _is_rank0() -> bool:
    return not dist.is_initialized() or dist.get_rank() == 0


class CheckpointManager(Configurable):
    @dataclass(kw_only=True, slots=True)
    class Config(Configurable.Config):
        enable: bool = False
        folder: str = "checkpoint"
        interval: int = 500
        initial_load_path: str | None = None
        initial_load_model_only: bool = True
        initial_load_in_hf: bool = False
        last_save_model_only: bool = True
        last_save_in_hf: bool = False
        export_dtype: Literal["float16", "bfloat16", "float32"] = "float32"
        async_mode: Literal["disabled", "async", "async_with_pinned_mem"] = "disabled"
        keep_latest_k: int = 10
        load_step: int = -1
        exclude_from_loading: list[str] = field(default_factory=list)
        fallback_on_load_error: bool = True
        """Resuming from the latest step: if that checkpoint cannot be read (a truncated or
        corrupt shard, a missing file), try the next older one instead of failing."""
        enable_first_step_checkpoint: bool = False
        create_seed_checkpoint: bool = False
        load_only: bool = False

    def __init__(self, config: Config, *, dataloader: Any = None, model_parts: list[nn.Module] | None = None,
                 optimizers: Any = None, lr_schedulers: Any = None, states: dict[str, Any] | None = None,
                 sd_adapter: Any = None, base_folder: str = "", **kw: Any):
        self.config = config
        self.enable = config.enable
        self.folder = os.path.join(base_folder, config.folder)
        self.sd_adapter = sd_adapter
        self.model_parts = model_parts or []
        self.states: dict[str, Any] = {}
        if model_parts is not None:
            self.states[MODEL] = ModelWrapper(model_parts)
        if optimizers is not None:
            self.states[OPTIMIZER] = optimizers
        if lr_schedulers is not None:
            self.states[LR_SCHEDULER] = lr_schedulers
        if dataloader is not None:
            self.states[DATALOADER] = dataloader
        self.states.update(states or {})
        self._pool = ThreadPoolExecutor(max_workers=1) if config.async_mode != "disabled" else None
        # Background saves run DCP's planning collectives while the next steps issue their own
        # NCCL collectives; on the default group the two threads could interleave differently on
        # different ranks. They get a dedicated gloo group instead (parity: the reference's
        # ``torchtitan/components/checkpoint.py:372,479-491``).
        self._async_pg = None
        if config.async_mode != "disabled" and config.enable and dist.is_initialized():
            self._async_pg = dist.new_group(backend="gloo")
        self._pending: Future | None = None
        self._purge_lock = threading.Lock()

    # ------------------------------------------------------------------ paths
    def _step_dir(self, step: int) -> str:
        return os.path.join(self.folder, f"step-{step}")

    def _existing_steps(self, folder: str | None = None) -> list[int]:
        folder = folder or self.folder
        if not os.path.isdir(folder):
            return []
        steps = []
        for d in os.listdir(folder):
            m = re.fullmatch(r"step-(\d+)", d)
            if m and os.path.exists(os.path.join(folder, d, ".metadata")):
                steps.append(int(m.group(1)))
        return sorted(steps)

    # ------------------------------------------------------------------- save
    def _should_save(self, step: int, last_step: bool) -> bool:
        if not self.enable or self.config.load_only:
            return False
        if step == 1 and self.config.enable_first_step_checkpoint:
            return True
        return last_step or step % self.config.interval == 0

    def _model_only_state(self) -> dict[str, Any]:
        sd = self.states[MODEL].state_dict()
        dt = TORCH_DTYPE_MAP[self.config.export_dtype]
        return {k: (v.to(dt) if torch.is_tensor(v) and v.is_floating_point() else v) for k, v in sd.items()}

    def save(self, step: int, last_step: bool = False) -> None:
        if not self._should_save(step, last_step):
            return
        self.maybe_wait_for_staging()
        t0 = time.perf_counter()
        path = self._step_dir(step)
        if last_step and self.config.last_save_model_only:
            state = self._model_only_state()
            if self.config.last_save_in_hf and self.sd_adapter is not None:
                self._save_hf(state, path)
            else:
                dcp.save(state, checkpoint_id=path)
        elif self._pool is not None:
            # Stage a host copy on this thread (the next step overwrites the device tensors), then
            # write it from the background thread over the gloo group.
            state = {k: v.state_dict() if hasattr(v, "state_dict") else v for k, v in self.states.items()}
            state = _to_pinned_host(state, pin=self.config.async_mode == "async_with_pinned_mem", copy_cpu=True)
            self._pending = self._pool.submit(dcp.save, state, checkpoint_id=path, process_group=self._async_pg)
        else:
            dcp.save(self.states, checkpoint_id=path)
        logger.info(f"checkpoint step {step} issued in {time.perf_counter() - t0:.2f}s -> {path}")
        self._purge()

    def save_seed(self) -> str:
        """Write the freshly initialised model, full precision and model only, as step 0 (parity:
        the reference's ``--checkpoint.create_seed_checkpoint``).  A later run in the same dump
        folder, or any run given this step directory as ``initial_load_path``, starts from
        these weights whatever its own seed or parallel layout (DCP reshards on load)."""
        path = self._step_dir(0)
        dcp.save(self.states[MODEL].state_dict(), checkpoint_id=path)
        logger.info(f"seed checkpoint -> {path}")
        return path

    def _save_hf(self, state: dict[str, Any], path: str) -> None:
        from safetensors.torch import save_file

        full = {k: (v.full_tensor() if hasattr(v, "full_tensor") else v) for k, v in state.items()}
        hf = self.sd_adapter.to_hf(full)
        if _is_rank0():
            os.makedirs(path, exist_ok=True)
            save_file({k: v.contiguous().cpu() for k, v in hf.items()}, os.path.join(path, "model.safetensors"))

    def maybe_wait_for_staging(self) -> None:
        if self._pending is not None:
            self._pending.result()
            self._pending = None

    def _purge(self) -> None:
        k = self.config.keep_latest_k
        if k <= 0 or not _is_rank0():
            return
        with self._purge_lock:
            for s in self._existing_steps()[:-k]:
                shutil.rmtree(self._step_dir(s), ignore_errors=True)

    # ------------------------------------------------------------------- load
    def load(self, step: int = -1) -> bool:
        if not self.enable:
            return False
        c = self.config
        steps = self._existing_steps()
        if not steps:
            if c.initial_load_path:
                return self._initial_load(c.initial_load_path)
            return False
        candidates = sorted(steps, reverse=True) if step == -1 else [step]
        if step != -1 or not c.fallback_on_load_error:
            candidates = candidates[:1]
        keys = [k for k in self.states if k not in c.exclude_from_loading]
        errors = []
        for s in candidates:
            path = self._step_dir(s)
            try:
                if not os.path.exists(os.path.join(path, ".metadata")):
                    raise FileNotFoundError(f"no checkpoint at {path}")
                if s == 0:  # a seed checkpoint holds the model's weights alone
                    sd = self.states[MODEL].state_dict()
                    dcp.load(sd, checkpoint_id=path)
                    self.states[MODEL].load_state_dict(sd)
                    logger.info(f"loaded seed checkpoint from {path}")
                    return True
                dcp.load({k: self.states[k] for k in keys}, checkpoint_id=path)
            except (Exception, CheckpointException) as e:  # noqa: BLE001 - reported, then an older step is tried
                errors.append(f"step {s}: {type(e).__name__}: {e}")
                if len(candidates) > 1:
                    logger.warning(f"checkpoint step {s} could not be loaded ({type(e).__name__}: {e}); "
                                   "trying an older one")
                continue
            logger.info(f"loaded checkpoint step {s} from {path} (keys {keys})")
            return True
        raise RuntimeError("no loadable checkpoint: " + "; ".join(errors))

    def _initial_load(self, path: str) -> bool:
        if self.config.initial_load_in_hf:
            from safetensors.torch import load_file

            files = sorted(f for f in os.listdir(path) if f.endswith(".safetensors"))
            hf = {}
            for f in files:
                hf.update(load_file(os.path.join(path, f)))
            native = self.sd_adapter.from_hf(hf)
            self.states[MODEL].load_state_dict(native)
        else:
            sd = self.states[MODEL].state_dict()
            dcp.load(sd if self.config.initial_load_model_only else {MODEL: sd}, checkpoint_id=path)
            self.states[MODEL].load_state_dict(sd)
        logger.info(f"initial weights loaded from {path}")
        return True

    def close(self) -> None:
        self.maybe_wait_for_staging()
        if self._pool is not None:
            self._pool.shutdown(wait=True)


def _to_pinned_host(obj: Any, pin: bool = True, copy_cpu: bool = False) -> Any:
    """Host copy of a (nested) state dict: device tensors (and, with ``copy_cpu``, host
    tensors too) are copied into fresh, optionally pinned, host buffers. DTensors keep their
    global shape and stride, which matters for uneven shards (dim 0 not divisible by the
    mesh size), where the shape inferred from the local piece would be wrong."""
    if torch.is_tensor(obj):
        is_dt = hasattr(obj, "to_local")
        local = obj.to_local() if is_dt else obj
        if local.is_cuda or copy_cpu:
            h = torch.empty(local.shape, dtype=local.dtype, pin_memory=pin and local.is_cuda)
            h.copy_(local, non_blocking=local.is_cuda)
            if local.is_cuda:
                torch.cuda.current_stream().synchronize()
            if is_dt:
                from torch.distributed.tensor import DTensor

                return DTensor.from_local(h, obj.device_mesh, obj.placements, run_check=False,
                                          shape=obj.shape, stride=obj.stride())
            return h
        return obj
    if isinstance(obj, dict):
        return {k: _to_pinned_host(v, pin, copy_cpu) for k, v in obj.items()}
    if isinstance(obj, list):
        return [_to_pinned_host(v, pin, copy_cpu) for v in obj]
    return obj
