"""Pipeline parallelism over ``torch.distributed.pipelining`` (NCCL p2p).

Stage construction (behaviour parity: ``torchtitan/distributed/pipeline_parallel.py:47-507``):
the number of virtual stages is ``pp`` x {1 for single-stage schedules, 2 for
multi-stage} or ``ceil((L + first_less + last_less) / layers_per_stage)``; the
embedding and the norm+output head count as ``first_less``/``last_less``
layer-equivalents when layers are split; every stage is a deep copy of the
meta model with the layers (and embedding / head) it does not own deleted, so
FQNs stay global; stages are placed round-robin (``loop``) or in V order for
``ZBVZeroBubble``/``DualPipeV``; each stage is parallelized with the model's
``parallelize_fn``.
"""
from __future__ import annotations

import copy
import math
from typing import Any

import torch
import torch.nn as nn

from torchtitan_b200.utils.logging import logger


def generate_llm_fqn_per_model_part(num_stages: int, num_layers: int, input_weight: int = 1,
                                    output_weight: int = 1, first: str = "tok_embeddings",
                                    last: tuple[str, ...] = ("norm", "output")) -> list[list[str]]:
    """Split ``num_layers`` decoder layers (+ embedding / head weights) evenly into stages."""
    if num_stages < 1:
        raise ValueError("num_stages must be >= 1")
    if num_stages == 1:
        return [[first] + [f"layers.{i}" for i in range(num_layers)] + list(last)]
    total = num_layers + input_weight + output_weight
    base, extra = divmod(total, num_stages)
    sizes = [base + (1 if s < extra else 0) for s in range(num_stages)]
    parts: list[list[str]] = []
    layer = 0
    for s, size in enumerate(sizes):
        names: list[str] = []
        budget = size
        if s == 0:
            names.append(first)
            budget -= input_weight
        if s == num_stages - 1:
            budget -= output_weight
        if budget < 0 or (budget == 0 and 0 < s < num_stages - 1):
            raise ValueError(f"stage {s} would hold no layers; use fewer stages")
        for _ in range(max(budget, 0)):
            if layer < num_layers:
                names.append(f"layers.{layer}")
                layer += 1
        if s == num_stages - 1:
            while layer < num_layers:
                names.append(f"layers.{layer}")
                layer += 1
            names += list(last)
        parts.append(names)
    return parts


def stage_ids_this_rank(pp_rank: int, pp_size: int, num_stages: int, style: str = "loop") -> tuple[int, ...]:
    per = num_stages // pp_size
    if style == "loop":
        return tuple(pp_rank + s * pp_size for s in range(per))
    if style == "v":
        assert per == 2
        return (pp_rank, num_stages - 1 - pp_rank)
    raise ValueError(style)


def _prune(model: nn.Module, keep: list[str]) -> nn.Module:
    m = copy.deepcopy(model)
    keep_layers = {n.split(".", 1)[1] for n in keep if n.startswith("layers.")}
    for k in list(m.layers.keys()):
        if k not in keep_layers:
            del m.layers[k]
    first = getattr(model, "pp_first_module", "tok_embeddings")
    last = tuple(getattr(model, "pp_last_modules", ("norm", "output")))
    for attr in (first, *last):
        if attr not in keep and getattr(m, attr, None) is not None:
            setattr(m, attr, None)
    return m


def get_schedule_class(name: str):
    from torch.distributed.pipelining.schedules import get_schedule_class as g

    return g(name)


def pipeline_llm(model: nn.Module, *, parallel_dims: Any, training: Any, parallelism: Any, ac_config: Any,
                 device: torch.device, parallelize_fn: Any, loss_fn: Any, model_converters: Any = None,
                 compile_config: Any = None, dump_folder: str = "", model_config: Any = None, **_: Any):
    from torch.distributed.pipelining import PipelineStage
    from torch.distributed.pipelining.schedules import PipelineScheduleSingle

    pp_mesh = parallel_dims.get_mesh("pp")
    sched_cls = get_schedule_class(parallelism.pipeline_parallel_schedule)
    single = issubclass(sched_cls, PipelineScheduleSingle)
    n_layers = len(model.layers)
    lps = parallelism.pipeline_parallel_layers_per_stage
    iw, ow = parallelism.pipeline_parallel_first_stage_less_layers, parallelism.pipeline_parallel_last_stage_less_layers
    if lps is not None:
        n_stages = math.ceil((n_layers + iw + ow) / lps)
        if n_stages % parallel_dims.pp:
            raise ValueError(f"{n_stages} virtual stages not divisible by pp={parallel_dims.pp}")
    else:
        n_stages = parallel_dims.pp * (1 if single else 2)
    per_rank = n_stages // parallel_dims.pp
    if single and per_rank != 1:
        raise ValueError("single-stage schedule needs exactly one stage per rank")
    if not single and per_rank < 2:
        raise ValueError("multi-stage schedule needs >= 2 stages per rank")
    fqns = parallelism.module_fqns_per_model_part or generate_llm_fqn_per_model_part(
        n_stages, n_layers, iw, ow, getattr(model, "pp_first_module", "tok_embeddings"),
        tuple(getattr(model, "pp_last_modules", ("norm", "output"))))
    style = "v" if parallelism.pipeline_parallel_schedule in ("ZBVZeroBubble", "DualPipeV") else "loop"
    pp_rank = pp_mesh.get_local_rank()
    stages, parts = [], []
    for sid in stage_ids_this_rank(pp_rank, parallel_dims.pp, n_stages, style):
        part = _prune(model, fqns[sid])
        part = parallelize_fn(part, parallel_dims=parallel_dims, training=training, model_converters=model_converters,
                              parallelism=parallelism, compile_config=compile_config, ac_config=ac_config,
                              dump_folder=dump_folder)
        stages.append(PipelineStage(part, sid, n_stages, device, group=pp_mesh.get_group()))
        parts.append(part)
        logger.info(f"PP rank {pp_rank} stage {sid}: {fqns[sid]}")
    n_mb = training.local_batch_size // parallelism.pipeline_parallel_microbatch_size
    if n_mb < 1:
        raise ValueError("local_batch_size must be >= pipeline_parallel_microbatch_size")
    lpb = getattr(model, "attn_res_layers_per_block", None)
    if lpb and style == "loop" and parallelism.pipeline_parallel_attnres_cache:
        from torchtitan_b200.models.common.attn_res import setup_stage_cache

        sids = list(stage_ids_this_rank(pp_rank, parallel_dims.pp, n_stages, style))
        setup_stage_cache(parts, sids, fqns, parallel_dims.pp, n_mb, lpb)
    if single:
        sched = sched_cls(stages[0], n_microbatches=n_mb, loss_fn=loss_fn, scale_grads=False)
    else:
        sched = sched_cls(stages, n_microbatches=n_mb, loss_fn=loss_fn, scale_grads=False)
    if parallelism.pipeline_parallel_schedule_csv:
        sched._load_csv(parallelism.pipeline_parallel_schedule_csv)
    first = any(s.is_first for s in stages)
    last = any(s.is_last for s in stages)
    return sched, parts, first, last
