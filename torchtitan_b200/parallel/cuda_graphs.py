"""CUDA-graph capture of transformer blocks, this framework's replacement for the
reference's per-block ``torch.compile`` and its graph trainer's cudagraph pass
(``distributed/compile.py:27-149``, ``experiments/graph_trainer/cudagraph.py``).

Each dense decoder block's forward and backward are captured once
(``torch.cuda.make_graphed_callables``) for the step's fixed activation shape and
replayed every step: one graph launch per block and direction instead of one
launch per kernel, with the kernels and their arguments fixed in the graph.

Requirements, checked before capture:
* parameters keep their storage between steps: one GPU, the peer-memory data
  parallel runtime, or replicated DDP-style weights; not FSDP2 (it re-materialises
  parameters every step), and no tensor/context/pipeline/expert parallelism
  (their collectives and host-side routing are outside the graph);
* MoE blocks only with the fused routing kernel and without forced load balancing: then
  routing, the padded expert layout and the grouped GEMMs run without a device-to-host
  read (the PyTorch routing fallback sizes ``bincount`` on the host);
* fixed shapes: the graphs are captured for ``[local_batch_size, seq_len, dim]``;
  the RoPE tables are read from the model's buffers at fixed addresses.
Gradients leave the graphed backward through the normal AccumulateGrad nodes, so
gradient hooks (the peer runtime's bucket copies) run unchanged.
"""
from __future__ import annotations

from typing import Any

import torch
import torch.nn as nn

from torchtitan_b200.utils.logging import logger


class _Call(nn.Module):
    """The captured function: the block's own forward with the RoPE tables bound."""

    def __init__(self, forward, params: list[nn.Parameter], cos: torch.Tensor, sin: torch.Tensor):
        super().__init__()
        self._fwd = forward
        self._params = params
        self.cos, self.sin = cos, sin

    def parameters(self, recurse: bool = True):
        return iter(self._params)

    def forward(self, h):
        return self._fwd(h, self.cos, self.sin, None)


def _graphed_forward(orig, graphed, shape, cos, sin):
    """Replays the graphs for the captured case (training, grad enabled, same shape, same
    RoPE tables, no masks) and runs the block's own forward otherwise."""

    def forward(h, c, s, attention_masks=None):
        if (torch.is_grad_enabled() and attention_masks is None and tuple(h.shape) == shape
                and c.data_ptr() == cos.data_ptr() and s.data_ptr() == sin.data_ptr()):
            return graphed(h)
        return orig(h, c, s, attention_masks)

    return forward


def cuda_graphs_applicable(parallel_dims: Any, model: nn.Module) -> str | None:
    """None if the model can be captured, else the reason it cannot."""
    pd = parallel_dims
    if not torch.cuda.is_available():
        return "CUDA graphs need a GPU"
    if pd.tp_enabled or pd.cp_enabled or pd.pp_enabled or pd.ep_enabled:
        return "tensor/context/pipeline/expert parallelism is not captured"
    if getattr(model, "_dp_runtime", None) is None and pd.dp_enabled and \
            any(type(p).__name__ == "DTensor" for p in model.parameters()):
        return "FSDP2 re-materialises parameters every step"
    if not hasattr(model, "layers") or not hasattr(model, "rope"):
        return "only decoder models with model.layers and RoPE tables are captured"
    for blk in model.layers.values():
        moe = getattr(blk, "moe", None)
        if moe is not None:
            from torchtitan_b200.models.common.moe import _router_kernel_enabled

            if not _router_kernel_enabled() or getattr(moe.router, "force_load_balance", False):
                return "MoE routing without the fused routing kernel reads expert counts on the host"
    return None


def apply_cuda_graphs(model: nn.Module, batch: int, seq: int, dtype: torch.dtype, warmup: int = 3) -> int:
    """Capture every block of ``model.layers`` for ``[batch, seq, dim]`` inputs.  Returns the
    number of captured blocks."""
    dev = next(model.parameters()).device
    cos, sin = model.rope.tables(seq, None)
    dim = model.tok_embeddings.weight.shape[1]
    n = 0
    for blk in model.layers.values():
        orig = blk.forward
        call = _Call(orig, list(blk.parameters()), cos, sin)
        sample = torch.randn(batch, seq, dim, device=dev, dtype=dtype, requires_grad=True)
        graphed = torch.cuda.make_graphed_callables(call, (sample,), num_warmup_iters=warmup)
        # the module tree (and so every checkpoint name) stays as it is: only forward changes
        blk.forward = _graphed_forward(orig, graphed, (batch, seq, dim), cos, sin)
        n += 1
    torch.cuda.synchronize(dev)
    logger.info(f"captured {n} blocks in CUDA graphs for [{batch}, {seq}, {dim}] {dtype}")
    return n
