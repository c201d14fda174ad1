"""SimpleFSDP: data parallelism written as per-parameter functional collectives, so a traced
training step shows every all-gather / reduce-scatter / all-reduce as a graph node that the
graph passes can bucket, reorder and duplicate.

Parity target: ``experiments/graph_trainer/simple_fsdp.py:261-329`` (``data_parallel`` with
``replicate`` / ``fully_shard`` / ``hybrid_shard``, ``MixedPrecisionPolicy``,
``disable_active_parametrization``).

Storage: each parameter becomes a DTensor on the data-parallel mesh (``Shard(0)`` on the
shard dim, ``Replicate()`` on a replicate dim), so optimizers, grad-norm clipping and DCP
checkpoints see ordinary sharded DTensors.  Compute: reading ``module.<name>`` returns the
full tensor built by :class:`_GatherParam` from the LOCAL shard:

  forward   cast to ``param_dtype`` -> pad dim 0 to the even shard size -> all_gather (shard
            dim) -> drop the padding rows
  backward  cast to ``reduce_dtype`` -> pad -> reduce_scatter(sum) (shard dim) ->
            all_reduce(sum) (replicate dim) -> drop padding -> cast to the shard's dtype

Both directions use ``torch.distributed._functional_collectives``, whose ops
(``_c10d_functional.all_gather_into_tensor`` + ``wait_tensor`` ...) survive ``make_fx``.
Gradients are SUMS over ranks (the trainer normalises the loss by the global token count).

The attribute read is intercepted by swapping the module's class for a cached subclass with
one property per parameter; ``state_dict`` / ``named_parameters`` read ``_parameters``
directly and still see the DTensor shards.  Tensor-parallel DTensor parameters are not
composed with this wrapper (``NotImplementedError``).
"""
from __future__ import annotations

import contextlib
import sys
from dataclasses import dataclass
from typing import Iterator

import torch
import torch.distributed._functional_collectives as funcol
import torch.nn as nn
from torch.distributed.tensor import DTensor, Replicate, Shard, distribute_tensor

_ACTIVE = True


@contextlib.contextmanager
def disable_active_parametrization() -> Iterator[None]:
    """Inside this context ``module.<param>`` returns the stored DTensor shard (for weight
    initialisation, inspection and checkpoint conversion) instead of gathering it."""
    global _ACTIVE
    prev, _ACTIVE = _ACTIVE, False
    try:
        yield
    finally:
        _ACTIVE = prev


@dataclass(frozen=True)
class MixedPrecisionPolicy:
    param_dtype: torch.dtype | None = None
    """dtype of the gathered compute weight (None: the stored dtype)."""
    reduce_dtype: torch.dtype | None = None
    """dtype the gradient is reduced in (None: the compute dtype)."""
    fp8_all_gather_modules: tuple[type, ...] = ()
    """Parameters (2-D and up) of modules of these types are all-gathered as FP8 E4M3 codes with
    one fp32 scale per row (448 / row amax), half the bytes of bf16, and dequantized to
    ``param_dtype`` after the gather.  Rows never straddle ranks, so no cross-rank amax is needed."""


def _fp8_rows(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Rowwise E4M3 codes (as uint8) and inverse scales of a [rows, ...] tensor."""
    xf = x.float().reshape(x.shape[0], -1)
    scale = 448.0 / xf.abs().amax(1).clamp_min(1e-12)
    codes = (xf * scale[:, None]).to(torch.float8_e4m3fn).view(torch.uint8)
    return codes, (1.0 / scale)


class _GatherParam(torch.autograd.Function):
    @staticmethod
    def forward(ctx, local, spec: "_DPSpec"):
        ctx.spec = spec
        ctx.local_dtype = local.dtype
        ctx.local_rows = local.shape[0] if local.dim() else 0
        x = local if spec.param_dtype is None else local.to(spec.param_dtype)
        if spec.shard_group is None:
            return x.clone() if x is local else x
        if spec.fp8 and x.dim() >= 2:
            codes, inv = _fp8_rows(local)
            pad = spec.shard_rows - codes.shape[0]
            if pad:
                codes = torch.nn.functional.pad(codes, (0, 0, 0, pad))
                inv = torch.nn.functional.pad(inv, (0, pad))
            codes = funcol.all_gather_tensor(codes.contiguous(), 0, spec.shard_group)[: spec.full_rows]
            inv = funcol.all_gather_tensor(inv.contiguous(), 0, spec.shard_group)[: spec.full_rows]
            full = codes.view(torch.float8_e4m3fn).float() * inv[:, None]
            return full.to(x.dtype).reshape((spec.full_rows,) + tuple(x.shape[1:]))
        pad = spec.shard_rows - x.shape[0]
        if pad:
            x = torch.nn.functional.pad(x, (0, 0) * (x.dim() - 1) + (0, pad))
        full = funcol.all_gather_tensor(x.contiguous(), 0, spec.shard_group)
        return full[: spec.full_rows] if spec.full_rows != full.shape[0] else full

    @staticmethod
    def backward(ctx, g):
        spec: _DPSpec = ctx.spec
        rd = spec.reduce_dtype or g.dtype
        g = g.to(rd).contiguous()
        if spec.shard_group is not None:
            pad = spec.shard_rows * spec.shard_size - g.shape[0]
            if pad:
                g = torch.nn.functional.pad(g, (0, 0) * (g.dim() - 1) + (0, pad))
            g = funcol.reduce_scatter_tensor(g, "sum", 0, spec.shard_group)
            if ctx.local_rows != g.shape[0]:
                g = g[: ctx.local_rows]
        if spec.replicate_group is not None:
            g = funcol.all_reduce(g, "sum", spec.replicate_group)
        return g.to(ctx.local_dtype), None


@dataclass(frozen=True, eq=False)
class _DPSpec:
    shard_group: object | None
    replicate_group: object | None
    shard_size: int
    shard_rows: int
    full_rows: int
    param_dtype: torch.dtype | None
    reduce_dtype: torch.dtype | None
    fp8: bool = False


def _gather(stored: torch.Tensor, spec: _DPSpec) -> torch.Tensor:
    local = stored.to_local() if isinstance(stored, DTensor) else stored
    return _GatherParam.apply(local, spec)


_SUBCLASSES: dict[tuple[type, tuple[str, ...]], type] = {}


def _make_property(name: str) -> property:
    def get(self):
        stored = self._parameters[name]
        if not _ACTIVE or stored is None:
            return stored
        return _gather(stored, self._simple_fsdp_specs[name])

    return property(get)


def _wrap_class(mod: nn.Module, names: tuple[str, ...]) -> None:
    key = (type(mod), names)
    cls = _SUBCLASSES.get(key)
    if cls is None:
        cls = type(f"SimpleFSDP{type(mod).__name__}", (type(mod),), {n: _make_property(n) for n in names})
        # importable under its own name, so pickling a module (or a traced graph) finds it
        cls.__module__ = __name__
        setattr(sys.modules[__name__], cls.__name__, cls)
        _SUBCLASSES[key] = cls
    mod.__class__ = cls


def data_parallel(model: nn.Module, device_mesh, mode: str = "fully_shard",
                  mp_policy: MixedPrecisionPolicy | None = None) -> nn.Module:
    """Shard (``fully_shard``), replicate (``replicate``) or replicate-then-shard on a 2-D mesh
    (``hybrid_shard``: mesh dims ``[replicate, shard]``) every parameter of ``model`` in place.
    Parameters may live on the meta device (materialise with ``to_empty`` + init under
    :func:`disable_active_parametrization` afterwards)."""
    mp = mp_policy or MixedPrecisionPolicy()
    if mode == "fully_shard":
        placements, shard_dim, rep_dim = (Shard(0),), 0, None
    elif mode == "replicate":
        placements, shard_dim, rep_dim = (Replicate(),), None, 0
    elif mode == "hybrid_shard":
        if device_mesh.ndim != 2:
            raise ValueError("hybrid_shard needs a 2-D mesh [replicate, shard]")
        placements, shard_dim, rep_dim = (Replicate(), Shard(0)), 1, 0
    else:
        raise ValueError(f"unknown SimpleFSDP mode {mode!r}")
    if device_mesh.ndim != len(placements):
        raise ValueError(f"mode {mode} needs a {len(placements)}-D mesh, got {device_mesh.ndim}-D")
    shard_size = device_mesh.size(shard_dim) if shard_dim is not None else 1
    # a mesh dim of one rank moves nothing: no collective is issued for it
    shard_group = device_mesh.get_group(shard_dim) if shard_dim is not None and shard_size > 1 else None
    rep_group = device_mesh.get_group(rep_dim) if rep_dim is not None and device_mesh.size(rep_dim) > 1 else None
    for mod in list(model.modules()):
        if type(mod).__name__.startswith("SimpleFSDP"):
            continue
        names = []
        specs = {}
        for name, p in list(mod.named_parameters(recurse=False)):
            if p is None:
                continue
            if isinstance(p, DTensor):
                raise NotImplementedError("SimpleFSDP over tensor-parallel DTensor parameters is not composed")
            rows = p.shape[0] if p.dim() else 1
            if p.dim() == 0:
                raise ValueError(f"SimpleFSDP cannot shard 0-d parameter {name}")
            if p.device.type == "meta":
                per = -(-rows // shard_size)
                r = device_mesh.get_local_rank(shard_dim) if shard_dim is not None else 0
                mine = max(0, min(per, rows - r * per)) if shard_dim is not None else rows
                dt = DTensor.from_local(torch.empty((mine,) + tuple(p.shape[1:]), dtype=p.dtype, device="meta"),
                                        device_mesh, placements, run_check=False, shape=p.shape, stride=p.stride())
            else:
                dt = distribute_tensor(p.data, device_mesh, placements)
            mod.register_parameter(name, nn.Parameter(dt, requires_grad=p.requires_grad))
            fp8 = bool(mp.fp8_all_gather_modules) and isinstance(mod, mp.fp8_all_gather_modules) and p.dim() >= 2
            specs[name] = _DPSpec(shard_group, rep_group, shard_size, -(-rows // shard_size), rows,
                                  mp.param_dtype, mp.reduce_dtype, fp8)
            names.append(name)
        if names:
            mod._simple_fsdp_specs = specs
            _wrap_class(mod, tuple(names))
    model._simple_fsdp_mesh = device_mesh
    return model


def is_simple_fsdp(model: nn.Module) -> bool:
    return getattr(model, "_simple_fsdp_mesh", None) is not None


def dp_group_size(model: nn.Module) -> int:
    mesh = getattr(model, "_simple_fsdp_mesh", None)
    return 1 if mesh is None else mesh.size()


def local_parameters(model: nn.Module) -> list[tuple[str, nn.Parameter]]:
    """(FQN, stored parameter) in ``named_parameters`` order: the leaves a traced step takes
    as inputs and returns gradients for."""
    return [(n, p) for n, p in model.named_parameters() if p.requires_grad]

