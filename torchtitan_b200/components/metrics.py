"""Training metrics: device-timed throughput, MFU, memory; TB/W&B sinks.

Parity with ``torchtitan/components/metrics.py:261-582`` (tps, tflops, mfu,
loss avg/max, grad norm, memory, data-loading share), with one deliberate
difference: step time is measured on the device with CUDA events bracketing
each logged interval and reduced as the MAX over ranks, so throughput is
what the slowest rank achieved (the reference uses host ``perf_counter``).
"""
from __future__ import annotations

import os
import time
from collections import namedtuple
from dataclasses import dataclass
from typing import Any

import torch
import torch.distributed as dist

from torchtitan_b200.config import Configurable
from torchtitan_b200.utils.device import Color, NoColor, get_peak_flops
from torchtitan_b200.utils.logging import logger

DeviceMemStats = namedtuple("DeviceMemStats", "max_active_gib max_active_pct max_reserved_gib max_reserved_pct "
                                              "num_alloc_retries num_ooms")


class DeviceMemoryMonitor:
    def __init__(self, device: str | torch.device = "cuda"):
        self.cuda = torch.cuda.is_available() and str(device).startswith("cuda")
        if self.cuda:
            self.device = torch.device(device)
            self.device_name = torch.cuda.get_device_name(self.device)
            self.capacity = torch.cuda.get_device_properties(self.device).total_memory
            torch.cuda.reset_peak_memory_stats()
        else:
            self.device, self.device_name, self.capacity = torch.device("cpu"), "cpu", 1

    def get_peak_stats(self) -> DeviceMemStats:
        if not self.cuda:
            return DeviceMemStats(0, 0, 0, 0, 0, 0)
        s = torch.cuda.memory_stats(self.device)
        gib = 1024 ** 3
        act, res = s.get("active_bytes.all.peak", 0), s.get("reserved_bytes.all.peak", 0)
        return DeviceMemStats(act / gib, 100 * act / self.capacity, res / gib, 100 * res / self.capacity,
                              s.get("num_alloc_retries", 0), s.get("num_ooms", 0))

    def reset_peak_stats(self) -> None:
        if self.cuda:
            torch.cuda.reset_peak_memory_stats()


class BaseLogger:
    def log(self, metrics: dict[str, Any], step: int) -> None:
        pass

    def close(self) -> None:
        pass


class TensorBoardLogger(BaseLogger):
    def __init__(self, log_dir: str):
        from torch.utils.tensorboard import SummaryWriter

        self.w = SummaryWriter(log_dir, max_queue=1000)

    def log(self, metrics, step):
        for k, v in metrics.items():
            self.w.add_scalar(k, v, step)

    def close(self):
        self.w.close()


class WandBLogger(BaseLogger):
    def __init__(self, log_dir: str, config_dict: dict | None = None):
        import wandb

        self.wandb = wandb
        self.run = wandb.init(project=os.getenv("WANDB_PROJECT", "torchtitan_b200"), dir=log_dir,
                              config=config_dict, mode=os.getenv("WANDB_MODE", "offline"))

    def log(self, metrics, step):
        self.run.log(metrics, step=step)

    def close(self):
        self.run.finish()


class JsonlLogger(BaseLogger):
    """One JSON object per logged step (``{"step": N, <metric>: value, ...}``): the format
    ``torchtitan_b200.loss_compare`` reads."""

    def __init__(self, path: str):
        os.makedirs(os.path.dirname(path), exist_ok=True)
        self.f = open(path, "a")

    def log(self, metrics, step):
        import json

        self.f.write(json.dumps({"step": step, **{k: float(v) for k, v in metrics.items()}}) + "\n")
        self.f.flush()

    def close(self):
        self.f.close()


class _Fanout(BaseLogger):
    def __init__(self, loggers):
        self.loggers = loggers

    def log(self, metrics, step):
        for lg in self.loggers:
            lg.log(metrics, step)

    def close(self):
        for lg in self.loggers:
            lg.close()


class MetricsProcessor(Configurable):
    @dataclass(kw_only=True, slots=True)
    class Config(Configurable.Config):
        log_freq: int = 10
        enable_tensorboard: bool = False
        disable_color_printing: bool = False
        save_tb_folder: str = "tb"
        save_for_all_ranks: bool = False
        enable_wandb: bool = False
        enable_jsonl: bool = False
        """Append every logged step to ``<dump_folder>/<save_tb_folder>/rank_<r>/metrics.jsonl``."""

    def __init__(self, config: Config, *, parallel_dims: Any = None, dump_folder: str = "./outputs",
                 pp_schedule: str = "1F1B", config_dict: dict | None = None, has_quantization: bool = False,
                 device: str | torch.device = "cuda", **kw: Any):
        self.config = config
        self.parallel_dims = parallel_dims
        self.has_quantization = has_quantization
        self.device_memory_monitor = DeviceMemoryMonitor(device if torch.cuda.is_available() else "cpu")
        self.color = NoColor() if config.disable_color_printing else Color()
        self.gpu_peak_flops = get_peak_flops(self.device_memory_monitor.device_name)
        self.num_flops_per_token = 0.0
        self.ntokens_since_last_log = 0
        self.data_loading_times: list[float] = []
        self.optimizers = self.model_parts = None
        self.logger: BaseLogger = BaseLogger()
        rank = dist.get_rank() if dist.is_initialized() else 0
        if config.save_for_all_ranks or rank == 0:
            d = os.path.join(dump_folder, config.save_tb_folder, f"rank_{rank}")
            loggers: list[BaseLogger] = []
            if config.enable_tensorboard:
                loggers.append(TensorBoardLogger(d))
            elif config.enable_wandb:
                loggers.append(WandBLogger(d, config_dict))
            if config.enable_jsonl:
                loggers.append(JsonlLogger(os.path.join(d, "metrics.jsonl")))
            if loggers:
                self.logger = loggers[0] if len(loggers) == 1 else _Fanout(loggers)
        self._t_host = time.perf_counter()
        self._ev_start = self._new_event()
        self.last_metrics: dict[str, float] = {}

    @staticmethod
    def _new_event():
        if torch.cuda.is_available():
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            return e
        return None

    def should_log(self, step: int) -> bool:
        return step == 1 or step % self.config.log_freq == 0

    def _interval_seconds(self) -> float:
        """Device time since the previous log, MAX over ranks."""
        if self._ev_start is not None:
            end = torch.cuda.Event(enable_timing=True)
            end.record()
            end.synchronize()
            dt = self._ev_start.elapsed_time(end) / 1e3
            self._ev_start = end
        else:
            now = time.perf_counter()
            dt, self._t_host = now - self._t_host, now
        t = torch.tensor([dt], dtype=torch.float64,
                         device="cuda" if torch.cuda.is_available() and dist.is_initialized()
                         and dist.get_backend() == "nccl" else "cpu")
        if dist.is_initialized() and dist.get_world_size() > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def log(self, step: int, global_avg_loss: float, global_max_loss: float, grad_norm: float,
            extra_metrics: dict[str, Any] | None = None) -> None:
        dt = max(self._interval_seconds(), 1e-9)
        pd = self.parallel_dims
        non_dp = (pd.cp * pd.tp * pd.pp) if pd is not None else 1
        tps = self.ntokens_since_last_log / (dt * non_dp)
        tflops = self.num_flops_per_token * tps / 1e12
        mfu = 100 * self.num_flops_per_token * tps / self.gpu_peak_flops
        mem = self.device_memory_monitor.get_peak_stats()
        dl = sum(self.data_loading_times)
        m = {
            "loss_metrics/global_avg_loss": float(global_avg_loss),
            "loss_metrics/global_max_loss": float(global_max_loss),
            "grad_norm": float(grad_norm),
            "throughput(tps)": tps,
            "tflops": tflops,
            "mfu(%)": mfu,
            "time_metrics/end_to_end(s)": dt / max(1, self.config.log_freq),
            "time_metrics/data_loading(s)": dl / max(1, len(self.data_loading_times)),
            "time_metrics/data_loading(%)": 100 * dl / dt,
            "memory/max_active(GiB)": mem.max_active_gib,
            "memory/max_reserved(GiB)": mem.max_reserved_gib,
            "memory/max_reserved(%)": mem.max_reserved_pct,
            "memory/num_alloc_retries": mem.num_alloc_retries,
            "memory/num_ooms": mem.num_ooms,
        }
        if self.has_quantization:
            m.pop("mfu(%)")
        if extra_metrics:
            m.update({k: float(v) if torch.is_tensor(v) else v for k, v in extra_metrics.items()})
        self.logger.log(m, step)
        self.last_metrics = m
        c = self.color
        logger.info(
            f"{c.red}step: {step:2}  {c.green}loss: {global_avg_loss:8.5f}  {c.cyan}grad_norm: {grad_norm:7.4f}  "
            f"{c.yellow}memory: {mem.max_reserved_gib:5.2f}GiB({mem.max_reserved_pct:.2f}%)  "
            f"{c.blue}tps: {round(tps):,}  {c.cyan}tflops: {tflops:,.2f}  "
            + (f"{c.magenta}mfu: {mfu:.2f}%{c.reset}" if not self.has_quantization else c.reset)
        )
        self.ntokens_since_last_log = 0
        self.data_loading_times.clear()
        self.device_memory_monitor.reset_peak_stats()

    def close(self) -> None:
        self.logger.close()
