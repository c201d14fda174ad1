"""Data parallelism with replicated compute weights and a sharded optimizer
(ZeRO-2 layout), communicating through the ranks' own memory over NVLink.

What the reference does with FSDP2 on a pure data-parallel mesh
(``models/llama3/infra/parallelize.py`` ``apply_fsdp`` over ``dp_shard``/``dp_replicate``,
``distributed/parallel_dims.py``) this runtime does with a different split of
work, chosen for a node of 8 GPUs with 180 GB each:

* the bf16 compute weights are replicated (an 8B model is 16 GB), so the
  forward and backward issue no parameter all-gathers at all;
* the fp32 masters and Adam moments are sharded 1/W per rank;
* gradients are bucketed in backward order.  When a bucket is complete, one
  kernel (``dp_reduce_scatter_bucket``) signals the peers, waits (bounded) for
  theirs, and sums this rank's slice of every peer's bf16 bucket with P2P loads
  into an fp32 shard gradient — transfer and reduction are the same pass, on a
  side stream, overlapping the rest of backward;
* the fused AdamW updates the fp32 shard and stores the new bf16 weights
  straight into every rank's weight buffer (the all-gather is the optimizer's
  epilogue), followed by a cross-GPU epoch barrier.

Buffers are symmetric allocations (``torch.distributed._symmetric_memory``):
one flat bf16 weight buffer, one flat bf16 gradient buffer and a flag array per
rank, mapped into every peer.  On CPU (gloo, tests) the same runtime runs with
``comm="collective"``: all-reduce / all-gather replace the peer kernels, and
everything else — layout, hooks, buckets, optimizer, checkpoint — is shared.
"""
from __future__ import annotations

import dataclasses
import os
from typing import Any

import torch
import torch.distributed as dist
import torch.nn as nn

_ALIGN = 64  # elements: every parameter and every shard starts on a 128-byte boundary


@dataclasses.dataclass
class Bucket:
    index: int
    offset: int  # element offset in the flat buffers
    length: int  # padded: a multiple of _ALIGN * world
    params: list[int]
    pending: int = 0
    launched: bool = False

    def shard_len(self, world: int) -> int:
        return self.length // world


def plan_layout(numels: list[int], world: int, bucket_elems: int, align: int = _ALIGN):
    """Pack parameters (given in backward order) into buckets of about
    ``bucket_elems`` elements.  Returns (offsets, buckets, total_elems)."""
    offsets: list[int] = []
    buckets: list[Bucket] = []
    cur: list[int] = []
    start = pos = 0

    def close():
        nonlocal start, pos, cur
        unit = align * world
        length = -(-(pos - start) // unit) * unit
        buckets.append(Bucket(len(buckets), start, length, cur))
        start = pos = start + length
        cur = []

    for i, n in enumerate(numels):
        pos = -(-pos // align) * align
        offsets.append(pos)
        pos += n
        cur.append(i)
        if pos - start >= bucket_elems:
            close()
    if cur:
        close()
    return offsets, buckets, start


def peer_dp_applicable(parallel_dims: Any, training: Any, parallelism: Any) -> bool:
    """Pure data parallelism on one node of CUDA devices with bf16 compute over fp32 masters."""
    mode = getattr(parallelism, "data_parallel_comm", "auto")
    if mode == "fsdp2" or parallel_dims.world_size < 2 or getattr(parallel_dims, "semi_sync_replicas", False):
        return False
    pure_dp = not (parallel_dims.tp_enabled or parallel_dims.cp_enabled or parallel_dims.pp_enabled
                   or parallel_dims.ep_enabled)
    if mode == "peer":
        if not pure_dp:
            raise ValueError("data_parallel_comm='peer' supports pure data parallelism only")
        return True
    one_node = int(os.environ.get("LOCAL_WORLD_SIZE", parallel_dims.world_size)) == parallel_dims.world_size
    # 8 ranks: a run of the 8B bench stalled at its second step (cause not yet found), so
    # ``auto`` keeps FSDP2 there; ``peer`` still selects this runtime explicitly
    return (pure_dp and one_node and parallel_dims.world_size <= 4 and torch.cuda.is_available()
            and training.mixed_precision_param == "bfloat16" and training.dtype == "float32"
            and not training.enable_cpu_offload)


def apply_peer_dp(model: nn.Module, dp_mesh: Any, bucket_mb: int = 256) -> nn.Module:
    """Mark ``model``; the trainer calls :func:`materialize_data_parallel` after weight init."""
    model._peer_dp_spec = (dp_mesh, bucket_mb)
    return model


class PeerDataParallel:
    def __init__(self, model: nn.Module, dp_mesh: Any, *, bucket_mb: int = 256, comm: str | None = None,
                 compute_dtype: torch.dtype | None = None):
        if getattr(dp_mesh, "ndim", 1) > 1:
            dp_mesh = dp_mesh._flatten()
        self.flat_mesh = dp_mesh
        self.group = dp_mesh.get_group()
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        seen: set[int] = set()
        params = []
        for p in model.parameters():
            if p.requires_grad and id(p) not in seen:
                seen.add(id(p))
                params.append(p)
        params.reverse()  # registration order reversed ~ the order backward produces gradients
        self.params = params
        dev = params[0].device
        self.device = dev
        self.comm = comm or ("peer" if dev.type == "cuda" else "collective")
        self.dtype = compute_dtype or (torch.bfloat16 if dev.type == "cuda" else torch.float32)
        if self.comm == "peer" and self.dtype != torch.bfloat16:
            raise ValueError("peer data parallelism runs bf16 compute weights")
        elem = torch.empty((), dtype=self.dtype).element_size()
        self.offsets, self.buckets, self.total = plan_layout([p.numel() for p in params], self.world,
                                                             bucket_mb * 2**20 // elem)
        self.shard_total = self.total // self.world
        self.epoch = 0
        # a wait for the other ranks gives up after this long (error code readable by check())
        self.wait_limit_s = float(os.environ.get("TTB_DP_WAIT_S", "20"))
        self.sync = True
        self._got: list[bool] = []
        self._next_launch = 0
        self._first_micro = True
        self._stream = torch.cuda.Stream(dev) if dev.type == "cuda" else None
        self._alloc_buffers()
        self._init_weights()
        self.grad_shard = torch.zeros(self.shard_total, dtype=torch.float32, device=dev)
        self._hooks = [p.register_post_accumulate_grad_hook(self._make_hook(i)) for i, p in enumerate(params)]
        self._bucket_of = {}
        for b in self.buckets:
            for i in b.params:
                self._bucket_of[i] = b
        self.barrier()

    # ------------------------------------------------------------ buffers
    def _alloc_buffers(self) -> None:
        dev, n = self.device, self.total
        if self.comm == "peer":
            # these buffers are read and written with plain peer loads/stores only
            os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")
            from torch.distributed import _symmetric_memory as symm

            from torchtitan_b200.ops._ext import ext

            self._ext = ext()
            from .watchdog import install

            self.watchdog = install(self._ext)
            name = self.group.group_name
            self.wbuf = symm.empty(n, dtype=torch.bfloat16, device=dev)
            self.gbuf = symm.empty(n, dtype=torch.bfloat16, device=dev)
            self.flags = symm.empty((len(self.buckets) + 1) * self.world, dtype=torch.int32, device=dev)
            self.gbuf.zero_()
            self.flags.zero_()
            hw, hg, hf = (symm.rendezvous(t, name) for t in (self.wbuf, self.gbuf, self.flags))
            self._handles = (hw, hg, hf)
            self.w_ptrs = [int(x) for x in hw.buffer_ptrs]
            self.g_ptrs = [int(x) for x in hg.buffer_ptrs]
            self.f_ptrs = [int(x) for x in hf.buffer_ptrs]
            torch.cuda.synchronize(dev)
            dist.barrier(group=self.group)
        else:
            self.wbuf = torch.zeros(n, dtype=self.dtype, device=dev)
            self.gbuf = torch.zeros(n, dtype=self.dtype, device=dev)

    @torch.no_grad()
    def _init_weights(self) -> None:
        """Rank 0's initial weights everywhere; fp32 master shards cut from them."""
        src = dist.get_global_rank(self.group, 0)
        self.master = torch.empty(self.shard_total, dtype=torch.float32, device=self.device)
        r = self.rank
        for b in self.buckets:
            full = torch.zeros(b.length, dtype=torch.float32, device=self.device)
            for i in b.params:
                p = self.params[i]
                val = p.data.float().contiguous()
                dist.broadcast(val, src=src, group=self.group)
                o = self.offsets[i] - b.offset
                full[o:o + p.numel()].copy_(val.view(-1))
            sl = b.shard_len(self.world)
            self.master[b.offset // self.world:b.offset // self.world + sl].copy_(full[r * sl:(r + 1) * sl])
            self.wbuf[b.offset:b.offset + b.length].copy_(full)
        for i, p in enumerate(self.params):
            o = self.offsets[i]
            p.data = self.wbuf[o:o + p.numel()].view(p.shape)

    # ------------------------------------------------------------ backward
    def begin_step(self, n_microbatches: int) -> None:
        self._micro_left = n_microbatches
        self._first_micro = True
        self._got = [False] * len(self.params)
        for b in self.buckets:
            b.pending = len(b.params)
            b.launched = False
        self._next_launch = 0

    def begin_microbatch(self, index: int, count: int) -> None:
        if index == 0:
            self.begin_step(count)
        self._first_micro = index == 0
        self.sync = index == count - 1
        if not self._first_micro:
            for b in self.buckets:
                b.pending = len(b.params)

    def _make_hook(self, i: int):
        def hook(p: torch.Tensor) -> None:
            g = p.grad
            o = self.offsets[i]
            view = self.gbuf[o:o + p.numel()]
            with torch.no_grad():
                if self._first_micro:
                    view.copy_(g.reshape(-1))
                else:
                    view.add_(g.reshape(-1))
            p.grad = None
            self._got[i] = True
            if self.sync:
                b = self._bucket_of[i]
                b.pending -= 1
                if b.pending == 0:
                    self._launch_ready()
        return hook

    def _launch_ready(self) -> None:
        """Launch complete buckets strictly in bucket-index order.  Every rank then issues the
        same sequence of waiting kernels on its reduction stream whatever order its autograd
        engine produced the gradients in: a rank waiting on bucket k never sits behind a
        kernel for bucket j > k that a peer has queued after its own bucket k."""
        while self._next_launch < len(self.buckets) and self.buckets[self._next_launch].pending == 0:
            self._launch(self.buckets[self._next_launch])
            self._next_launch += 1

    def _launch(self, b: Bucket) -> None:
        if b.launched:
            return
        b.launched = True
        sl = b.shard_len(self.world)
        out = self.grad_shard[b.offset // self.world:b.offset // self.world + sl]
        if self.comm == "peer":
            cur = torch.cuda.current_stream(self.device)
            self._stream.wait_stream(cur)
            with torch.cuda.stream(self._stream):
                self._ext.dp_reduce_scatter_bucket(self.g_ptrs, self.f_ptrs, self.rank, b.offset, b.length, out,
                                                   1.0, b.index, self.epoch + 1, 64, self.wait_limit_s)
        else:
            full = self.gbuf[b.offset:b.offset + b.length].float()
            dist.all_reduce(full, group=self.group)
            out.copy_(full[self.rank * sl:(self.rank + 1) * sl])

    def finish_backward(self) -> None:
        """Launch any bucket whose parameters got no gradient (in bucket order on every rank)
        and make the current stream wait for the reductions."""
        for b in self.buckets:
            if not b.launched:
                for i in b.params:  # parameters without a gradient this step contribute zeros
                    if not self._got[i]:
                        o = self.offsets[i]
                        self.gbuf[o:o + self.params[i].numel()].zero_()
                self._launch(b)
        self._next_launch = len(self.buckets)
        if self._stream is not None:
            torch.cuda.current_stream(self.device).wait_stream(self._stream)

    def grad_sumsq(self) -> torch.Tensor:
        """Global sum of squared gradient entries (for norm clipping), as a device scalar."""
        if self.comm == "peer":
            sq = self._ext.multi_sumsq([self.grad_shard])
        else:
            sq = self.grad_shard.pow(2).sum()
        dist.all_reduce(sq, group=self.group)
        return sq

    # ------------------------------------------------------------ optimizer side
    def shard_views(self, t: torch.Tensor) -> list[torch.Tensor]:
        return [t[b.offset // self.world:b.offset // self.world + b.shard_len(self.world)] for b in self.buckets]

    @torch.no_grad()
    def adamw_step(self, m: torch.Tensor, v: torch.Tensor, *, lr: float, beta1: float, beta2: float, eps: float,
                   weight_decay: float, step: int, clip: tuple[torch.Tensor, float] | None) -> None:
        clip_total, clip_max = clip if clip is not None else (None, 0.0)
        self.finish_backward()
        if self.comm == "peer":
            ps, gs, ms, vs = (self.shard_views(t) for t in (self.master, self.grad_shard, m, v))
            offs = [b.offset + self.rank * b.shard_len(self.world) for b in self.buckets]
            self._ext.adamw(ps, gs, ms, vs, float(lr), float(beta1), float(beta2), float(eps), float(weight_decay),
                            int(step), [], clip_total.float().reshape(()).contiguous() if clip_total is not None
                            else None, float(clip_max), peer_offsets=offs, peer_bases=self.w_ptrs)
            self.epoch += 1
            self.barrier()
        else:
            from torchtitan_b200 import ops

            ops.fused_adamw_([self.master], [self.grad_shard], [m], [v], lr=lr, beta1=beta1, beta2=beta2, eps=eps,
                             weight_decay=weight_decay, step=step, clip_total=clip_total, clip_max=clip_max)
            self.epoch += 1
            self.gather_weights()

    @torch.no_grad()
    def gather_weights(self) -> None:
        """Rewrite every rank's compute weights from the fp32 master shards."""
        for b, shard in zip(self.buckets, self.shard_views(self.master)):
            out = self.wbuf[b.offset:b.offset + b.length]
            if self.comm == "peer":
                # one-off path (checkpoint load): NCCL into this rank's own buffer
                dist.all_gather_into_tensor(out, shard.to(self.dtype), group=self.group)
            else:
                parts = [torch.empty_like(shard) for _ in range(self.world)]
                dist.all_gather(parts, shard, group=self.group)
                out.copy_(torch.cat(parts).to(self.dtype))

    @torch.no_grad()
    def masters_from_weights(self) -> None:
        """After compute weights were loaded from outside (a model-only checkpoint):
        cut the fp32 master shards from them."""
        for b, shard in zip(self.buckets, self.shard_views(self.master)):
            sl = b.shard_len(self.world)
            shard.copy_(self.wbuf[b.offset + self.rank * sl:b.offset + (self.rank + 1) * sl])

    def barrier(self) -> None:
        if self.comm == "peer":
            self.epoch_barrier_count = getattr(self, "epoch_barrier_count", 0) + 1
            self._ext.dp_barrier(self.f_ptrs, self.rank, len(self.buckets), self.epoch_barrier_count,
                                 limit_s=self.wait_limit_s)
        else:
            dist.barrier(group=self.group)

    def check(self) -> None:
        """Raise if a peer wait gave up (a rank stopped answering) since the last check."""
        wd = getattr(self, "watchdog", None)
        if wd is not None and wd.poll() is not None:
            from .watchdog import describe

            raise RuntimeError(f"peer data parallel: {describe(wd.error)}")
        if self.comm == "peer":
            info = self._ext.dp_error_info()
            code = self._ext.dp_error_code(True)
            if code:
                raise RuntimeError(f"peer data parallel: a wait for the other ranks timed out (code {code}; slot "
                                   f"{info[0]}, epoch {info[1]}, source rank {info[2]}, flag seen {info[3]})")


@torch.no_grad()
def materialize_data_parallel(model: nn.Module) -> None:
    """After weight init: build the peer data-parallel runtime (if marked) or the
    single-replica fp32 masters."""
    spec = getattr(model, "_peer_dp_spec", None)
    if spec is not None:
        mesh, bucket_mb = spec
        model._dp_runtime = PeerDataParallel(model, mesh, bucket_mb=bucket_mb)
        return
    from torchtitan_b200.parallel.fsdp import materialize_replica_mixed_precision

    materialize_replica_mixed_precision(model)
