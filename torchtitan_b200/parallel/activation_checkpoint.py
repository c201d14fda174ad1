"""Activation checkpointing of transformer blocks.

Modes (parity: ``torchtitan/distributed/activation_checkpoint.py``):
  * ``full`` -- recompute the whole block in backward.
  * ``selective`` + ``selective_ac_option="op"`` -- per-op policy: keep the
    outputs of flash-attention forwards and of every second GEMM (the
    ``tt_b200::gemm`` custom op), keep reduce-scatter / all-to-all outputs,
    recompute everything else (norms, RoPE, SwiGLU are cheap on HBM3e).
    ``selective_ac_option="op_all_mm"`` keeps every GEMM output instead: no GEMM is
    recomputed, only the element-wise ops between them (about 10 GB more per GPU for
    Llama-3 8B at seq 8192, well inside 180 GB of HBM3e).
    GEMMs whose shapes match ``per_op_sac_force_recompute_mm_shapes_by_fqns``
    modules (e.g. the MoE router gate) are always recomputed.
  * ``selective`` + integer N -- full checkpointing of every N-th block.
"""
from __future__ import annotations

from collections import defaultdict
from typing import Any

import torch
import torch.nn as nn
from torch.distributed.algorithms._checkpoint.checkpoint_wrapper import checkpoint_wrapper
from torch.utils.checkpoint import CheckpointPolicy, create_selective_checkpoint_contexts

import torchtitan_b200.ops  # noqa: F401  (registers the custom ops)


def _save_list() -> set:
    s = {
        torch.ops.tt_b200.attn_fwd.default,
        torch.ops.aten._scaled_dot_product_efficient_attention.default,
        torch.ops.aten._scaled_dot_product_flash_attention.default,
        torch.ops._c10d_functional.reduce_scatter_tensor.default,
        torch.ops._c10d_functional.all_to_all_single.default,
        torch.ops.aten.max.default,
    }
    return s


def _op_sac_policy(force_recompute_shapes: set[tuple[int, int]], save_all_mm: bool = False):
    save = _save_list()
    gemm = torch.ops.tt_b200.gemm.default
    mm_ops = {gemm, torch.ops.aten.mm.default}

    def make():
        counts: dict[str, int] = defaultdict(int)

        def policy(ctx, func, *args, **kwargs):
            mode = "recompute" if ctx.is_recompute else "forward"
            if func in mm_ops:
                b = args[1]
                if tuple(b.shape) in force_recompute_shapes:
                    return CheckpointPolicy.PREFER_RECOMPUTE
                if save_all_mm:
                    return CheckpointPolicy.MUST_SAVE
                counts[f"{mode}_mm"] += 1
                # keep every second GEMM output
                return CheckpointPolicy.MUST_SAVE if counts[f"{mode}_mm"] % 2 == 1 else CheckpointPolicy.PREFER_RECOMPUTE
            return CheckpointPolicy.MUST_SAVE if func in save else CheckpointPolicy.PREFER_RECOMPUTE

        return create_selective_checkpoint_contexts(policy)

    return make


def _force_shapes(model: nn.Module, fqns: list[str]) -> set[tuple[int, int]]:
    shapes = set()
    for name, m in model.named_modules():
        if any(f in name for f in fqns) and hasattr(m, "weight") and m.weight is not None and m.weight.dim() == 2:
            shapes.add(tuple(m.weight.shape))
    return shapes


def _blocks(model: nn.Module):
    """(container, key, block) for every block: ``model.layers`` (a ModuleDict), or each
    ModuleDict/ModuleList a model lists in ``ac_block_containers`` (e.g. FLUX's double
    and single stream blocks)."""
    for cont in getattr(model, "ac_block_containers", None) or [model.layers]:
        items = list(cont.items()) if isinstance(cont, nn.ModuleDict) else list(enumerate(cont))
        for k, blk in items:
            yield cont, k, blk


def apply_ac(model: nn.Module, ac: Any, **_: Any) -> None:
    if ac.mode == "none":
        return
    if ac.mode == "full":
        for cont, k, blk in _blocks(model):
            cont[k] = checkpoint_wrapper(blk, preserve_rng_state=ac.preserve_rng_state)
        return
    if ac.mode == "memory_budget":
        raise NotImplementedError("memory_budget AC needs a tracing compiler; use 'selective' or 'full'")
    opt = ac.selective_ac_option
    if opt in ("op", "op_all_mm"):
        make_ctx = _op_sac_policy(_force_shapes(model, ac.per_op_sac_force_recompute_mm_shapes_by_fqns),
                                  save_all_mm=opt == "op_all_mm")
        for cont, k, blk in _blocks(model):
            cont[k] = checkpoint_wrapper(blk, context_fn=make_ctx, preserve_rng_state=ac.preserve_rng_state)
        return
    every = int(opt)
    if every <= 0:
        raise ValueError("selective_ac_option must be 'op' or a positive integer")
    for i, (cont, k, blk) in enumerate(_blocks(model)):
        if i % every == 0:
            cont[k] = checkpoint_wrapper(blk, preserve_rng_state=ac.preserve_rng_state)
