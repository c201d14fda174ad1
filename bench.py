"""Flagship benchmark: Llama-3 8B, FSDP2, bf16, seq 8192, local batch 1, per-op SAC, AdamW.

  python bench.py --gpus N --steps K --warmup W [--impl ours|reference]

For N > 1 it is launched with torchrun (one rank per GPU, NCCL).  W untimed
warm-up steps, then K timed steps bracketed by barrier + synchronize; the
device time (CUDA events) is reduced as the MAX over ranks.  A second timed
loop of K steps measures the same metric end to end through the public
``Trainer.train_step`` API with a host->device copy of each step's tokens
from pinned host memory and a device->host read of each step's loss.
Rank 0 prints one JSON line.  Data: synthetic uniform tokens; weights: random
init of the 8B architecture.  Inputs (16 GB of weights, 8192x128256 logits)
exceed the 126 MB L2, so no explicit flush is done between steps.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

BASELINE_TPS_PER_GPU = 8307.5  # reference, 8x B200 bf16, bs1 seq 8192, FSDP2 + SAC (docs/mxfp8.md:148-152)
# same table, quantized linears: mxfp8_cublas 9,969 and fp8 tensorwise 10,417 tokens/s (docs/mxfp8.md:153-155)
BASELINE_QUANT_TPS_PER_GPU = {"mxfp8": 9969.0, "float8": 10417.0}
METRIC = "tokens/sec (whole job) for Llama-3 8B FSDP2 bf16 training"


def _parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--seq-len", type=int, default=8192)
    ap.add_argument("--flavor", default="8B")
    ap.add_argument("--ac", default="selective")
    ap.add_argument("--dp-comm", default="auto", choices=["auto", "peer", "fsdp2"],
                    help="data-parallel runtime of this framework's arm (auto: peer memory on one node)")
    ap.add_argument("--sac-option", default="op_all_mm",
                    help="per-op SAC variant of this framework's arm: op_all_mm keeps every GEMM output")
    ap.add_argument("--quant", default="none", choices=["none", "mxfp8", "float8", "float8_rowwise"],
                    help="quantized linears (all but the output head), as the reference's converters")
    ap.add_argument("--profile-out", default=None, help="write a per-kernel time table of one extra step here")
    return ap.parse_args()


class ClockSampler:
    """Samples nvidia-smi clocks / throttle reasons in the background."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None

    def start(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                       "-i", str(self.gpu), "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.p = None

    def stop(self) -> dict:
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        self.p.wait(timeout=10)
        self.f.seek(0)
        rows = [r.split(", ") for r in self.f.read().strip().splitlines() if r.strip()]
        os.unlink(self.f.name)
        sm = [float(r[1]) for r in rows if len(r) >= 9 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if len(r) >= 9 and r[2].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            if len(r) < 9:
                continue
            for n, v in zip(names, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def _dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def _max_over_ranks(x: float) -> float:
    import torch
    import torch.distributed as dist

    if dist.is_initialized() and dist.get_world_size() > 1:
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())
    return x


def _count_launches(step_fn) -> int:
    """Kernels from this repo's extension launched by one step (names in namespace ttb)."""
    import torch

    with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA]) as prof:
        step_fn()
        torch.cuda.synchronize()
    n = 0
    for e in prof.events():
        if e.device_type == torch.autograd.DeviceType.CUDA and "ttb" in e.name:
            n += 1
    return n


def run_ours(a):
    import torch
    import torch.distributed as dist

    from torchtitan_b200.components.checkpoint import CheckpointManager
    from torchtitan_b200.components.metrics import MetricsProcessor
    from torchtitan_b200.config import ActivationCheckpointConfig, TrainingConfig
    from torchtitan_b200.models.llama3 import config_registry as reg
    from torchtitan_b200.models.llama3 import model_registry
    from torchtitan_b200.trainer import Trainer
    from torchtitan_b200.utils.logging import init_logger

    init_logger()
    rank, world, local = _dist_env()
    cfg = reg.llama3_8b()
    cfg.model_spec = model_registry(a.flavor)
    cfg.training = TrainingConfig(local_batch_size=1, seq_len=a.seq_len, steps=a.warmup + 2 * a.steps + 2,
                                  dtype="float32", mixed_precision_param="bfloat16")
    cfg.activation_checkpoint = ActivationCheckpointConfig(mode=a.ac, selective_ac_option=a.sac_option)
    cfg.metrics = MetricsProcessor.Config(log_freq=10 ** 9)
    cfg.checkpoint = CheckpointManager.Config(enable=False)
    cfg.validator.enable = False
    # where FSDP2 runs (8 ranks), keep the bf16 parameters gathered after the forward: 16 GB
    # per GPU buys back the backward's parameter all-gathers
    cfg.parallelism.fsdp_reshard_after_forward = os.environ.get("TTB_BENCH_RESHARD", "never")
    cfg.parallelism.data_parallel_comm = a.dp_comm
    if a.quant != "none":
        cfg.model_converters.names = [a.quant]
    trainer = Trainer(cfg)
    it = trainer.batch_generator(trainer.dataloader)
    tokens_per_step = cfg.training.local_batch_size * cfg.training.seq_len * trainer.dp_degree

    def step():
        trainer.step += 1
        return trainer.train_step(it)

    for _ in range(a.warmup):
        step()
    torch.cuda.synchronize()
    if dist.is_initialized():
        dist.barrier()
    clocks = ClockSampler(local)
    clocks.start()
    # ---- device-timed region
    torch.cuda.synchronize()
    if dist.is_initialized():
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(a.steps):
        loss = step()
    ev1.record()
    torch.cuda.synchronize()
    if dist.is_initialized():
        dist.barrier()
    torch.cuda.synchronize()
    dev_s = _max_over_ranks(ev0.elapsed_time(ev1) / 1e3)
    clk = clocks.stop()
    # ---- end-to-end region: public API, H2D of tokens (pinned) + D2H of the loss every step
    h2d = tokens_per_step // trainer.dp_degree * 8 * 2  # int64 inputs + labels per rank
    if dist.is_initialized():
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(a.steps):
        loss = step()
        _ = float(loss.item())
    torch.cuda.synchronize()
    e2e_s = _max_over_ranks(time.perf_counter() - t0)
    per_step_launches = _count_launches(step)
    if a.profile_out and rank == 0:
        with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA]) as prof:
            step()
            torch.cuda.synchronize()
        with open(a.profile_out, "w") as f:
            f.write(prof.key_averages().table(sort_by="cuda_time_total", row_limit=40, max_name_column_width=90))
    peak_mem = torch.cuda.max_memory_reserved() / 1024 ** 3
    value = tokens_per_step * a.steps / dev_s
    flops_tok = trainer.metrics_processor.num_flops_per_token
    mfu = 100 * value / world * flops_tok / 2.25e15
    out = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": a.steps,
        "warmup": a.warmup,
        "ms_per_step": round(1e3 * dev_s / a.steps, 2),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": (round(value / (BASELINE_TPS_PER_GPU * world), 4) if a.quant == "none"
                        else round(value / (BASELINE_QUANT_TPS_PER_GPU[a.quant] * world), 4)
                        if a.quant in BASELINE_QUANT_TPS_PER_GPU else None),
        "dtype": "bf16" if a.quant == "none" else f"{a.quant} linears (bf16 master weights, bf16 attention)",
        "data": "synthetic uniform tokens, random-init weights",
        "config": {"model": f"llama3_{a.flavor}", "global_batch": world, "seq_len": a.seq_len,
                   "parallelism": (f"dp{world} (replicated bf16 weights, sharded fp32 AdamW, peer-memory reduce-scatter"
                                   " and optimizer-fused all-gather)"
                                   if getattr(trainer.model_parts[0], "_dp_runtime", None) is not None
                                   else "single GPU (bf16 compute weights, fp32 masters in the fused AdamW; no sharding)"
                                   if world == 1
                                   else f"fsdp{world} (reshard_after_forward={cfg.parallelism.fsdp_reshard_after_forward})"), "ac": a.ac if a.ac != "selective" else f"selective ({a.sac_option})", "optimizer": "AdamW (fused, fp32 master)",
                   "l2": "inputs larger than L2 (no flush)", "quant": a.quant},
        "mfu_pct": round(mfu, 2),
        "tokens_per_sec_per_gpu": round(value / world, 1),
        "peak_mem_gib": round(peak_mem, 2),
        "clocks": clk,
        "e2e": {"value": round(tokens_per_step * a.steps / e2e_s, 1), "unit": "tokens/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4},
        "gpu_launches": per_step_launches * a.steps,
        "impl": "ours",
    }
    if rank == 0:
        print(json.dumps(out), flush=True)
    trainer.close()
    if dist.is_initialized():
        dist.destroy_process_group()


def _install_reference(ref):
    """Offline install of the reference source tree into ``ref`` (the same command the
    build notes record), for boxes where the git-ignored install was not carried over."""
    import shutil
    import subprocess

    src = os.environ.get("TTB_REFERENCE_SRC", "/root/reference")
    if not os.path.isdir(src):
        return
    subprocess.run([sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation",
                    "--no-deps", "--find-links", "/opt/wheelhouse", "--target", ref, src],
                   stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL, check=False)
    tok = os.path.join(src, "tests", "assets", "tokenizer")
    dst = os.path.join(ref, "assets", "tokenizer")
    if os.path.isdir(tok) and not os.path.isdir(dst):
        shutil.copytree(tok, dst)


def run_reference(a):
    if a.quant != "none":
        print(json.dumps({"impl": "reference", "unavailable": "the reference's Float8/MX converters need torchao, "
                          "which is not installed on this image"}))
        return
    here = os.path.dirname(os.path.abspath(__file__))
    ref = os.path.join(here, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "torchtitan")):
        _install_reference(ref)
    if not os.path.isdir(os.path.join(ref, "torchtitan")):
        print(json.dumps({"impl": "reference", "unavailable": "reference not installed under baseline/_ref"}))
        return
    sys.path.insert(0, ref)
    from baseline.reference_arm import run as ref_run

    ref_run(a, _dist_env, _max_over_ranks, ClockSampler, METRIC, BASELINE_TPS_PER_GPU)


if __name__ == "__main__":
    args = _parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)
