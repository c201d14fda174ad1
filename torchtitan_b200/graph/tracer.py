"""Trace a whole training step (forward + loss + backward) into ONE FX graph.

Parity target: the reference's ``aot_fx_trace`` mode (``experiments/graph_trainer/
make_fx_tracer.py``): non-strict ``make_fx`` tracing of forward, loss and backward, no
partitioner.  Here the traced function takes the LOCAL parameter tensors (the DTensor shards
of SimpleFSDP, or the plain parameters), the buffers, the batch and the token normaliser, and
returns ``[loss, grad_0, grad_1, ...]``; collectives appear as ``_c10d_functional`` nodes and
the sm_100a kernels as ``tt_b200`` / ``tt_b200_graph`` custom ops (:mod:`.traceable`).

Tracing runs under fake tensors (no kernel executes, no collective is issued); the graph is
then run eagerly node by node (optionally replayed as a CUDA graph, :mod:`.cudagraph`).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Callable

import torch
import torch.fx as fx
import torch.nn as nn
from torch.distributed.tensor import DTensor
from torch.fx.experimental.proxy_tensor import make_fx

from .traceable import traceable_kernels


@dataclass
class TracedStep:
    gm: fx.GraphModule
    param_names: list[str]
    buffer_names: list[str]
    n_params: int
    loss_node: str
    """name of the node holding the (normalised) loss: nodes after it are the backward."""
    meta: dict[str, Any] = field(default_factory=dict)

    def placeholder_param(self) -> dict[str, str]:
        """placeholder node name -> parameter FQN."""
        phs = [n for n in self.gm.graph.nodes if n.op == "placeholder"]
        return {phs[i].name: self.param_names[i] for i in range(self.n_params)}


def _local(t: torch.Tensor) -> torch.Tensor:
    return t.to_local() if isinstance(t, DTensor) else t


def step_inputs(model: nn.Module, param_names: list[str], buffer_names: list[str]):
    ps = dict(model.named_parameters())
    bs = dict(model.named_buffers())
    params = [_local(ps[n]).detach().requires_grad_(True) for n in param_names]
    buffers = [_local(bs[n]) for n in buffer_names]
    return params, buffers


def trace_train_step(model: nn.Module, loss_fn: Callable, inputs: torch.Tensor, labels: torch.Tensor,
                     norm: torch.Tensor, extra_kwargs: dict[str, torch.Tensor] | None = None) -> TracedStep:
    """``loss_fn(pred, labels)`` returns the summed loss; the traced loss is that sum / ``norm``.
    ``extra_kwargs`` (tensors, e.g. per-token positions and document ids of packed sequences)
    become trailing graph inputs in sorted-name order and are passed to the model by name."""
    param_names = [n for n, p in model.named_parameters() if p.requires_grad]
    buffer_names = [n for n, _ in model.named_buffers()]
    extra_names = sorted(extra_kwargs or {})

    def step(params, buffers, tokens, lbl, nrm, *extras):
        state = dict(zip(param_names, params))
        state.update(zip(buffer_names, buffers))
        pred = torch.func.functional_call(model, state, (tokens,), dict(zip(extra_names, extras)))
        loss = loss_fn(pred, lbl) / nrm
        grads = torch.autograd.grad(loss, params, allow_unused=True)
        return [loss] + [g if g is not None else torch.zeros_like(p) for g, p in zip(grads, params)]

    params, buffers = step_inputs(model, param_names, buffer_names)
    with traceable_kernels():
        gm = make_fx(step, tracing_mode="fake", _allow_non_fake_inputs=False)(
            params, buffers, inputs, labels, norm, *[extra_kwargs[n] for n in extra_names])
    out = next(n for n in gm.graph.nodes if n.op == "output")
    loss_node = out.args[0][0].name
    return TracedStep(gm, param_names, buffer_names, len(param_names), loss_node, {"extra_names": extra_names})


def backward_nodes(gm: fx.GraphModule, loss_node: str) -> set[fx.Node]:
    """Nodes traced after the loss (the backward), excluding the output node."""
    seen, out = False, set()
    for n in gm.graph.nodes:
        if seen and n.op != "output":
            out.add(n)
        if n.name == loss_node:
            seen = True
    return out


class GraphStepRunner:
    """Runs a traced step on the model's current local tensors and stores the gradients on
    the parameters (DTensor grads re-wrapped with the parameter's mesh and placements)."""

    def __init__(self, model: nn.Module, traced: TracedStep, executor: Callable | None = None):
        self.model = model
        self.traced = traced
        self.executor = executor or traced.gm
        ps = dict(model.named_parameters())
        self.params = [ps[n] for n in traced.param_names]
        bs = dict(model.named_buffers())
        self.buffers = [bs[n] for n in traced.buffer_names]
        self.copy_static_grads = True
        """With a CUDA-graph executor, copy the (static) gradient outputs before storing them:
        needed when a later microbatch of the same step replays the graph again."""

    @torch.no_grad()
    def __call__(self, inputs: torch.Tensor, labels: torch.Tensor, norm: torch.Tensor,
                 extra_kwargs: dict[str, torch.Tensor] | None = None) -> torch.Tensor:
        locs = [_local(p) for p in self.params]
        bufs = [_local(b) for b in self.buffers]
        names = self.traced.meta.get("extra_names", [])
        if sorted(extra_kwargs or {}) != names:
            raise ValueError(f"traced step takes extra inputs {names}, got {sorted(extra_kwargs or {})}")
        outs = self.executor(locs, bufs, inputs, labels, norm, *[extra_kwargs[n] for n in names])
        loss, grads = outs[0], outs[1:]
        static = getattr(self.executor, "outputs_are_static", False)
        for p, g in zip(self.params, grads):
            if static and p.grad is None and self.copy_static_grads:
                g = g.clone()  # the next replay overwrites the graph's output tensors
            if isinstance(p, DTensor):
                g = DTensor.from_local(g, p.device_mesh, p.placements, run_check=False, shape=p.shape,
                                       stride=p.stride())
            if p.grad is None:
                p.grad = g
            else:
                p.grad += g
        return loss.clone() if static else loss
