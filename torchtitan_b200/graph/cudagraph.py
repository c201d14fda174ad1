"""Replay a traced training step as one CUDA graph.

Parity target: ``experiments/graph_trainer/cudagraph.py`` (``CUDAGraphWrapper``: warm-up,
capture on first eligible call, static inputs, replay).  The traced step's inputs are the local
parameter tensors and buffers (stable storage: the optimizer updates them in place) plus the
batch; only the batch is copied into static buffers before each replay.  Outputs (loss and
gradients) are the graph's static tensors and are overwritten by the next replay, which the
step runner accounts for when gradients accumulate over microbatches.

A new input shape, device or parameter storage makes the executor fall back to eager
execution of the FX graph (and log it) instead of replaying a stale capture.
"""
from __future__ import annotations

from typing import Any

import torch
import torch.fx as fx

from torchtitan_b200.utils.logging import logger


class CUDAGraphExecutor:
    def __init__(self, gm: fx.GraphModule, warmup: int = 2):
        self.gm = gm
        self.warmup = warmup
        self.calls = 0
        self.graph: torch.cuda.CUDAGraph | None = None
        self.static_batch: list[torch.Tensor] = []
        self.static_out: Any = None
        self.key: tuple | None = None
        self.outputs_are_static = False

    @staticmethod
    def _key(params, buffers, batch) -> tuple:
        return (tuple(t.data_ptr() for t in params), tuple(t.data_ptr() for t in buffers),
                tuple((t.shape, t.dtype) for t in batch))

    def __call__(self, params, buffers, *batch):
        key = self._key(params, buffers, batch)
        if self.graph is not None and key == self.key:
            for s, b in zip(self.static_batch, batch):
                s.copy_(b, non_blocking=True)
            self.graph.replay()
            self.outputs_are_static = True
            return self.static_out
        if self.graph is not None:
            logger.warning("graph trainer: step inputs changed (shape or parameter storage); running eagerly")
            self.outputs_are_static = False
            return self.gm(params, buffers, *batch)
        self.calls += 1
        if self.calls <= self.warmup:
            self.outputs_are_static = False
            return self.gm(params, buffers, *batch)
        self.static_batch = [b.clone() for b in batch]
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            self.gm(params, buffers, *self.static_batch)  # allocator warm-up on the capture stream
        torch.cuda.current_stream().wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.static_out = self.gm(params, buffers, *self.static_batch)
        self.key = key
        self.graph.replay()
        self.outputs_are_static = True
        return self.static_out
