"""Async tensor parallelism on fused kernels: the sequence all-gather before a column-parallel
GEMM and the reduce-scatter after a row-parallel GEMM run inside ONE persistent tcgen05 GEMM
each (``csrc/tp_gemm.cu``), moving data over NVLink peer memory tile by tile:

* ``ag_matmul``: copy warps pull every peer's sequence shard into a local landing buffer while
  the GEMM starts on this rank's own rows; each remote chunk is consumed as soon as it has
  landed. The landing buffer is the gathered input the weight gradient needs.
* ``matmul_rs``: the GEMM computes the other ranks' output rows first and stores each partial
  tile straight into its owner's receive slot; the owner sums the ``tp`` partials of its rows.

Backward of one is the other (d/dx of AG->GEMM is GEMM->RS of the output gradient, and vice
versa); weight gradients are local GEMMs on the gathered tensors. The reference obtains the
same overlap from Inductor's micro-pipeline pass (``distributed/tensor_parallel.py:191-204``).

Buffers are symmetric allocations (``torch.distributed._symmetric_memory``) created on first
use of a shape, in the same order on every rank of the group (TP is SPMD). Only plain P2P loads
and stores are used (symmetric-memory multicast is switched off).
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from torchtitan_b200.ops._ext import ext

MAX_TP = 8


def fused_available(x: torch.Tensor, group) -> bool:
    if os.environ.get("TTB_TP_FUSED", "1") == "0" or not x.is_cuda or group is None:
        return False
    tp = dist.get_world_size(group)
    return 1 < tp <= MAX_TP and dist.get_backend(group) == "nccl"


class _GroupComm:
    def __init__(self, group):
        from torch.distributed import _symmetric_memory as symm

        os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")  # plain peer loads/stores only
        self.group = group
        self.tp, self.rank = dist.get_world_size(group), dist.get_rank(group)
        self.name = group.group_name
        self.symm = symm
        dev = torch.device("cuda", torch.cuda.current_device())
        self.dev = dev
        self.sig = symm.empty(2 * MAX_TP, dtype=torch.int32, device=dev)
        self.sig.zero_()
        self.done = symm.empty(2, dtype=torch.int32, device=dev)
        self.done.zero_()
        torch.cuda.synchronize(dev)
        self.sig_ptrs = [int(p) for p in symm.rendezvous(self.sig, self.name).buffer_ptrs]
        self.done_ptrs = [int(p) for p in symm.rendezvous(self.done, self.name).buffer_ptrs]
        self.epoch = 0
        self.rs_calls = 0
        self.shards: dict[tuple, tuple[torch.Tensor, list[int]]] = {}
        self.recvs: dict[tuple, tuple[torch.Tensor, list[int]]] = {}

    def _shard(self, rows: int, k: int):
        key = (rows, k)
        if key not in self.shards:
            t = self.symm.empty(rows, k, dtype=torch.bfloat16, device=self.dev)
            self.shards[key] = (t, [int(p) for p in self.symm.rendezvous(t, self.name).buffer_ptrs])
        return self.shards[key]

    def _recv(self, rows: int, n: int):
        key = (rows, n)
        if key not in self.recvs:
            t = self.symm.empty(2, self.tp, rows, n, dtype=torch.bfloat16, device=self.dev)
            self.recvs[key] = (t, [int(p) for p in self.symm.rendezvous(t, self.name).buffer_ptrs])
        return self.recvs[key]

    def ag_gemm(self, x2d: torch.Tensor, w: torch.Tensor, b_mn: bool) -> tuple[torch.Tensor, torch.Tensor]:
        """x2d [Ms, K] this rank's rows; w [N, K] (or [K, N] with ``b_mn``).
        Returns (D [tp*Ms, N], gathered input [tp*Ms, K])."""
        Ms, K = x2d.shape
        N = w.shape[1] if b_mn else w.shape[0]
        buf, ptrs = self._shard(Ms, K)
        buf.copy_(x2d)
        land = torch.empty(self.tp * Ms, K, dtype=torch.bfloat16, device=x2d.device)
        out = torch.empty(self.tp * Ms, N, dtype=torch.bfloat16, device=x2d.device)
        ready = torch.zeros(MAX_TP, dtype=torch.int32, device=x2d.device)
        self.epoch += 1
        ext().tp_gemm(0, ptrs, land, ready, out, w.contiguous(), b_mn, [], [], None, 0, self.sig_ptrs,
                      self.tp, self.rank, self.epoch, Ms, N, K)
        return out, land

    def gemm_rs(self, x2d: torch.Tensor, w: torch.Tensor, b_mn: bool) -> torch.Tensor:
        """x2d [tp*Ms, K] (chunk-major rows); returns this rank's reduced rows [Ms, N]."""
        M, K = x2d.shape
        Ms = M // self.tp
        N = w.shape[1] if b_mn else w.shape[0]
        recv, rptrs = self._recv(Ms, N)
        out = torch.empty(Ms, N, dtype=torch.bfloat16, device=x2d.device)
        parity = self.rs_calls % 2
        self.rs_calls += 1
        self.epoch += 1
        shards = [0] * self.tp
        x2d = x2d.contiguous()
        shards[self.rank] = x2d.data_ptr()
        ext().tp_gemm(1, shards, None, None, None, w.contiguous(), b_mn, rptrs, self.done_ptrs, out, parity,
                      self.sig_ptrs, self.tp, self.rank, self.epoch, Ms, N, K)
        return out


_COMMS: dict[str, _GroupComm] = {}


def _comm(group) -> _GroupComm:
    c = _COMMS.get(group.group_name)
    if c is None:
        c = _COMMS[group.group_name] = _GroupComm(group)
    return c


def shapes_ok(x: torch.Tensor, w_rows: int, k: int) -> bool:
    rows = x.numel() // x.shape[-1]
    return rows % 128 == 0 and w_rows % 32 == 0 and k % 64 == 0 and x.dtype == torch.bfloat16


def _chunk_major(x: torch.Tensor, tp: int) -> torch.Tensor:
    """[B, S, K] -> [tp * B * S/tp, K] with rank r's sequence slice of every batch row together."""
    B, S, K = x.shape
    if B == 1:
        return x.reshape(S, K)
    return x.view(B, tp, S // tp, K).transpose(0, 1).reshape(S * B, K)


def _from_chunk_major(y: torch.Tensor, B: int, tp: int) -> torch.Tensor:
    """[tp * B * s, N] chunk-major -> [B, tp * s, N]."""
    N = y.shape[-1]
    if B == 1:
        return y.view(1, -1, N)
    s = y.shape[0] // (tp * B)
    return y.view(tp, B, s, N).transpose(0, 1).reshape(B, tp * s, N)


class FusedAGMatmul(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, group):
        c = _comm(group)
        B = x.shape[0]
        y2d, land = c.ag_gemm(x.reshape(-1, x.shape[-1]), w, False)
        ctx.save_for_backward(land, w)
        ctx.group, ctx.B = group, B
        return _from_chunk_major(y2d, B, c.tp)

    @staticmethod
    def backward(ctx, dy):
        land, w = ctx.saved_tensors
        c = _comm(ctx.group)
        dy2d = _chunk_major(dy.contiguous(), c.tp)  # [tp*Ms, N]
        dx = c.gemm_rs(dy2d, w, True)                 # dy @ w, reduced to this rank's rows
        dw = ext().gemm(dy2d, land, True, True)       # dy^T @ x_gathered (rows in the same order)
        return dx.view(ctx.B, -1, dx.shape[-1]), dw.to(w.dtype), None


class FusedMatmulRS(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, group):
        c = _comm(group)
        B = x.shape[0]
        x2d = _chunk_major(x.contiguous(), c.tp)
        ctx.save_for_backward(x2d, w)
        ctx.group, ctx.B = group, B
        y = c.gemm_rs(x2d, w, False)
        return y.view(B, -1, y.shape[-1])

    @staticmethod
    def backward(ctx, dy):
        x2d, w = ctx.saved_tensors
        c = _comm(ctx.group)
        dx2d, dy_full = c.ag_gemm(dy.reshape(-1, dy.shape[-1]).contiguous(), w, True)  # gathered dy @ w
        dw = ext().gemm(dy_full, x2d, True, True)
        return _from_chunk_major(dx2d, ctx.B, c.tp), dw.to(w.dtype), None
