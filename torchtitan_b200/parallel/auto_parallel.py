"""AutoParallel: cost-based choice of the parallel layout for a model, a GPU count and a batch.

Parity target: ``experiments/autoparallel/llama3/parallelize_llama.py:26`` (the reference calls
the external ``autoparallel`` package, which solves an ILP over per-operator DTensor shardings
under a parameter-memory constraint).  This planner searches the layouts this framework's
appliers implement instead of per-operator placements: every factorisation of the GPU count
into ``dp_replicate x dp_shard x cp x tp`` (tp and cp within one NVSwitch node), sequence
parallelism, async (fused) TP, FSDP reshard-after-forward and the activation-checkpointing
mode.  Each candidate gets an analytic step time and a per-GPU memory estimate:

  compute   training FLOPs (6 N + attention, plus the recomputation of the AC mode) per GPU
            divided by the measured sustained bf16 GEMM rate x an efficiency that falls as
            TP shrinks the GEMMs
  FSDP      parameter all-gathers (bf16, once or twice) and fp32 gradient reduce-scatters over
            NVLink, hidden behind compute except for the part that exceeds it
  TP        per layer 4 activation collectives forward and 4 backward (SP: all-gather /
            reduce-scatter; no SP: all-reduce at twice the bytes); async TP hides most of it
  CP        ring attention K/V exchange per layer, overlapped with the attention tiles
  memory    fp32 master + grad + Adam moments over the sharding degree, gathered bf16
            weights, activations per token for the AC mode, logits; must fit the HBM budget

For 2-4 ranks of pure data parallelism the peer-memory runtime is a candidate too (replicated
bf16 weights and gradient buckets, sharded fp32 optimizer state; bf16 reduce-scatter and
weight stores over NVLink; no FSDP2 copy-in/copy-out passes).

The cheapest feasible candidate wins (ties go to fewer model-parallel dims).  Rates come from
``MEASURED_PEAKS.json`` when present (sustained GEMM TFLOP/s) and the pool's measured NVLink
peer-copy bandwidth otherwise.
"""
from __future__ import annotations

import json
import math
import os
from dataclasses import dataclass, field, replace
from typing import Any, Iterable

import torch.nn as nn

NVLINK_GBS = 770.0           # measured peer copy, GB/s per direction per GPU
HBM_BYTES = 180e9
GEMM_TFLOPS_FALLBACK = 1400.0  # sustained bf16, TFLOP/s


@dataclass(frozen=True)
class ModelShape:
    n_params: int
    n_embedding: int          # parameters outside the blocks' GEMMs (embedding rows)
    n_layers: int
    dim: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    vocab: int
    flops_per_token: float    # 6 N + attention, no recomputation


@dataclass(frozen=True)
class Hardware:
    gemm_tflops: float = GEMM_TFLOPS_FALLBACK
    hbm_gbs: float = 6500.0
    nvlink_gbs: float = NVLINK_GBS
    hbm_bytes: float = HBM_BYTES
    gpus_per_node: int = 8
    memory_fraction: float = 0.9
    peer_memory: bool = True
    """GPUs of one node reach each other's memory (the peer-memory data-parallel runtime)."""


@dataclass(frozen=True)
class Plan:
    dp_replicate: int
    dp_shard: int
    cp: int
    tp: int
    sequence_parallel: bool
    async_tp: bool
    reshard_after_forward: bool
    ac_mode: str
    grad_accum: int = 1
    dp_comm: str = "fsdp2"
    """``fsdp2`` or ``peer`` (replicated bf16 weights, sharded fp32 optimizer state, gradient
    reduce-scatter kernel and all-gather fused into AdamW over NVLink peer memory)."""
    step_s: float = 0.0
    memory_bytes: float = 0.0
    breakdown: dict = field(default_factory=dict, compare=False, hash=False)

    def describe(self) -> str:
        b = self.breakdown
        return (f"dp_replicate={self.dp_replicate} dp_shard={self.dp_shard} cp={self.cp} tp={self.tp} "
                f"sp={self.sequence_parallel} async_tp={self.async_tp} reshard={self.reshard_after_forward} "
                f"ac={self.ac_mode} ga={self.grad_accum} dp_comm={self.dp_comm}: {self.step_s * 1e3:.1f} ms/step, {self.memory_bytes / 2**30:.1f} GiB/GPU "
                f"(compute {b.get('compute', 0) * 1e3:.1f} ms, exposed comm {b.get('comm', 0) * 1e3:.1f} ms)")


def default_hardware() -> Hardware:
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                        "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            peaks = json.load(f)
        return Hardware(gemm_tflops=float(peaks.get("bf16_tflops_sustained") or GEMM_TFLOPS_FALLBACK),
                        hbm_gbs=float(peaks.get("hbm_gbs") or 6500.0))
    except (OSError, ValueError):
        return Hardware()


def model_shape(model: nn.Module, margs: Any, seq_len: int) -> ModelShape:
    """Shape summary of a (meta) model built from ``margs``."""
    n_params, fpt = margs.get_nparams_and_flops(model, seq_len)
    emb = sum(p.numel() for m in model.modules() if isinstance(m, nn.Embedding) for p in m.parameters())
    dim = int(getattr(margs, "dim", 0) or getattr(margs, "hidden_size", 0))
    n_heads = int(getattr(margs, "n_heads", 1))
    n_kv = int(getattr(margs, "n_kv_heads", None) or n_heads)
    head_dim = int(getattr(margs, "head_dim", 0) or (dim // max(n_heads, 1)))
    return ModelShape(n_params=int(n_params), n_embedding=int(emb), n_layers=int(getattr(margs, "n_layers", 1)),
                      dim=dim, n_heads=n_heads, n_kv_heads=n_kv, head_dim=head_dim,
                      vocab=int(getattr(margs, "vocab_size", 0)), flops_per_token=float(fpt))


def _divisors(n: int) -> list[int]:
    return [d for d in range(1, n + 1) if n % d == 0]


_RECOMPUTE = {"none": 1.0, "selective": 1.0 + 1.0 / 12, "full": 4.0 / 3.0}
# bf16 bytes kept per token per layer, in units of ``dim`` (flash attention: no S^2 term)
_ACT_BYTES_PER_DIM = {"none": 34.0, "selective": 22.0, "full": 2.0}


def estimate(shape: ModelShape, hw: Hardware, plan: Plan, global_batch: int, seq_len: int) -> Plan:
    """Fill in ``step_s``, ``memory_bytes`` and the breakdown of ``plan``."""
    world = plan.dp_replicate * plan.dp_shard * plan.cp * plan.tp
    dp = plan.dp_replicate * plan.dp_shard
    tokens_total = global_batch * seq_len
    tokens_dp = tokens_total / dp                 # tokens one TP/CP group processes per step
    tokens_mb = tokens_dp / plan.grad_accum       # ... per microbatch
    tokens_gpu_act = tokens_mb / plan.cp / (plan.tp if plan.sequence_parallel else 1)
    bw = hw.nvlink_gbs * 1e9

    eff = 0.78 * (0.94 ** math.log2(plan.tp)) * (0.97 ** math.log2(plan.cp))
    flops = shape.flops_per_token * tokens_total * _RECOMPUTE[plan.ac_mode] / world
    compute = flops / (hw.gemm_tflops * 1e12 * eff)

    p_local = shape.n_params / plan.tp           # parameters a TP rank holds before DP sharding
    fs = plan.dp_shard * plan.cp                 # FSDP shards over the data and context dims
    fsdp = 0.0
    hbm = hw.hbm_gbs * 1e9
    copies = 0.0  # memory passes of the data-parallel runtime itself (not hidden by overlap)
    if plan.dp_comm == "peer":
        frac = (fs - 1) / fs
        # bf16 gradient reduce-scatter per microbatch + bf16 weight stores fused into AdamW
        fsdp = p_local * frac * 2 / bw * plan.grad_accum + p_local * frac * 2 / bw
        copies = p_local * 2 * plan.grad_accum / hbm          # gradients into the bucket buffer
    elif fs > 1:
        frac = (fs - 1) / fs
        n_ag = 2 if plan.reshard_after_forward else 1
        # gathers and reductions repeat per microbatch
        fsdp = p_local * frac * (2 * n_ag + 4) / bw * plan.grad_accum
        # FSDP2 copy-in of the gathered bf16 parameters and copy-out of fp32 gradient shards
        copies = p_local * (2 * n_ag + 4) * plan.grad_accum / hbm
    if plan.dp_replicate > 1:
        frac = 2 * (plan.dp_replicate - 1) / plan.dp_replicate
        fsdp += p_local / fs * 4 * frac / bw
    tp_comm = 0.0
    if plan.tp > 1:
        act = tokens_dp / plan.cp * shape.dim * 2   # bf16 activations of one TP group, whole step
        frac = (plan.tp - 1) / plan.tp
        per = act * frac / bw * (1 if plan.sequence_parallel else 2)
        n = 8 + (4 if plan.ac_mode == "full" else 0)
        tp_comm = shape.n_layers * n * per
        if plan.async_tp:
            tp_comm *= 0.25
    cp_comm = 0.0
    if plan.cp > 1:
        kv = tokens_dp / plan.cp * 2 * shape.n_kv_heads * shape.head_dim * 2 / plan.tp
        cp_comm = shape.n_layers * 3 * kv * (plan.cp - 1) / bw * 0.3   # overlapped with the tiles
    exposed = max(0.0, fsdp - 0.85 * compute) + tp_comm + cp_comm + copies
    step = compute + exposed

    if plan.dp_comm == "peer":
        # fp32 master + Adam moments sharded; full bf16 weights and bf16 gradient buckets
        states = shape.n_params * 12 / fs + shape.n_params * 4
        gathered = 0.0
    else:
        states = shape.n_params * 16 / (fs * plan.tp)
        gathered = 2 * p_local * (2.0 / shape.n_layers if plan.reshard_after_forward else 1.0) if fs > 1 else 0.0
    acts = shape.n_layers * tokens_gpu_act * shape.dim * _ACT_BYTES_PER_DIM[plan.ac_mode]
    if plan.tp > 1 and not plan.sequence_parallel:
        acts = acts / plan.tp * 1.5  # head/hidden-sharded tensors shrink, replicated norms do not
    logits = tokens_mb / plan.cp * shape.vocab / plan.tp * 6
    mem = states + gathered + acts + logits + 3e9   # + workspace, allocator slack
    return replace(plan, step_s=step, memory_bytes=mem,
                   breakdown={"compute": compute, "comm": exposed, "fsdp": fsdp, "tp": tp_comm, "cp": cp_comm,
                              "states": states, "activations": acts})


def candidates(shape: ModelShape, hw: Hardware, world: int, global_batch: int, seq_len: int,
               ac_modes: Iterable[str] = ("none", "selective", "full"), allow_cp: bool = True) -> list[Plan]:
    out = []
    for tp in _divisors(world):
        if tp > hw.gpus_per_node or shape.n_heads % tp or shape.n_kv_heads % tp:
            continue
        for cp in _divisors(world // tp):
            if (cp > 1 and not allow_cp) or cp * tp > hw.gpus_per_node or seq_len % (2 * cp * tp):
                continue
            dp = world // (tp * cp)
            if global_batch % dp:
                continue
            for rep in _divisors(dp):
                shard = dp // rep  # rep > 1 with shard == 1 is pure replication (DDP)
                per_rank = global_batch // dp
                for sp in ((True, False) if tp > 1 else (False,)):
                    for atp in ((False, True) if tp > 1 and sp else (False,)):
                        for reshard in ((True, False) if shard * cp > 1 else (False,)):
                            for ac in ac_modes:
                                for ga in _divisors(per_rank):
                                    out.append(Plan(rep, shard, cp, tp, sp, atp, reshard, ac, ga))
                                    # peer-memory DP: pure data parallelism on one node, 2-4 ranks
                                    if hw.peer_memory and tp == cp == rep == 1 and 2 <= shard <= 4 and reshard:
                                        out.append(Plan(rep, shard, cp, tp, sp, atp, False, ac, ga, "peer"))
    return out


def plan_parallelism(shape: ModelShape, world: int, global_batch: int, seq_len: int,
                     hw: Hardware | None = None, **kw) -> list[Plan]:
    """All feasible plans, cheapest first.  Raises if nothing fits in memory."""
    hw = hw or default_hardware()
    budget = hw.hbm_bytes * hw.memory_fraction
    plans = [estimate(shape, hw, p, global_batch, seq_len) for p in candidates(shape, hw, world, global_batch,
                                                                                seq_len, **kw)]
    ok = [p for p in plans if p.memory_bytes <= budget]
    if not ok:
        best = min(plans, key=lambda p: p.memory_bytes) if plans else None
        raise ValueError(f"no parallel layout of {world} GPUs fits {budget / 2**30:.0f} GiB per GPU"
                         + (f" (smallest: {best.describe()})" if best else ""))
    return sorted(ok, key=lambda p: (round(p.step_s, 6), p.tp * p.cp, p.grad_accum, p.ac_mode != "none"))


def apply_plan(config: Any, plan: Plan) -> None:
    """Write ``plan`` into a trainer config (``parallelism`` and ``activation_checkpoint``)."""
    par = config.parallelism
    par.data_parallel_replicate_degree = plan.dp_replicate
    par.data_parallel_shard_degree = plan.dp_shard
    par.context_parallel_degree = plan.cp
    par.tensor_parallel_degree = plan.tp
    par.enable_sequence_parallel = plan.sequence_parallel
    par.enable_async_tensor_parallel = plan.async_tp
    par.fsdp_reshard_after_forward = "always" if plan.reshard_after_forward else "never"
    par.data_parallel_comm = plan.dp_comm
    config.activation_checkpoint.mode = plan.ac_mode


def auto_parallelize_config(config: Any, world: int) -> Plan:
    """Choose and apply the cheapest layout for ``config`` (model built on the meta device)."""
    import torch

    margs = config.model_spec.model
    with torch.device("meta"):
        model = margs.build()
    t = config.training
    dp_guess = world
    gbs = t.global_batch_size if t.global_batch_size > 0 else t.local_batch_size * dp_guess
    shape = model_shape(model, margs, t.seq_len)
    hw = default_hardware()
    if not torch.cuda.is_available():  # gloo / CPU runs: no peer memory
        hw = replace(hw, peer_memory=False)
    plans = plan_parallelism(shape, world, gbs, t.seq_len, hw=hw)
    best = plans[0]
    dp = best.dp_replicate * best.dp_shard
    # the global batch stays what the config implied; each data-parallel rank runs it in
    # ``grad_accum`` microbatches
    t.global_batch_size = gbs
    t.local_batch_size = gbs // dp // best.grad_accum
    apply_plan(config, best)
    return best


def main(argv: list[str] | None = None) -> list[Plan]:
    """``python -m torchtitan_b200.parallel.auto_parallel --ngpu 8 [--top 5] --module M --config C
    [--section.key value ...]``: print the cheapest feasible layouts for a registered config."""
    import argparse
    import sys

    import torch

    from torchtitan_b200.config.manager import ConfigManager

    p = argparse.ArgumentParser(description=main.__doc__.splitlines()[0])
    p.add_argument("--ngpu", type=int, default=8)
    p.add_argument("--top", type=int, default=5)
    args, rest = p.parse_known_args(sys.argv[1:] if argv is None else argv)
    cfg = ConfigManager().parse_args(rest)
    margs = cfg.model_spec.model
    with torch.device("meta"):
        model = margs.build()
    t = cfg.training
    gbs = t.global_batch_size if t.global_batch_size > 0 else t.local_batch_size * args.ngpu
    plans = plan_parallelism(model_shape(model, margs, t.seq_len), args.ngpu, gbs, t.seq_len)
    for i, plan in enumerate(plans[: args.top]):
        print(f"{i + 1}. {plan.describe()}")
    return plans


if __name__ == "__main__":
    main()
