"""Expert parallelism over NVLink peer memory (``expert_parallel_comm_backend="fused"``).

The NCCL path (``parallel.expert_parallel``) all-to-alls routed rows in
(source, expert) order, permutes them to expert order, pads them for the
grouped GEMM, and reverses all of it on the way back.  Here each source rank
stores its routed rows *directly* at their final position in the expert
owner's padded expert-major buffer (the layout the grouped tcgen05 GEMM
reads), and fetches expert outputs directly back into token order:

1. counts: every rank stores its ``[E]`` per-expert counts into every peer's
   ``[ep, E]`` matrix (one P2P row store), epoch barrier; the destination of every
   routed row is computed from the matrix on the device and the row stores of step 3
   are queued at once, while an asynchronous copy brings the matrix to pinned host
   memory; the host waits for that copy (the sizes of the padded expert buffer) only
   after the dispatch is in flight. The receive buffers are reserved once per batch
   shape for the worst case (all routed rows of all ranks on one owner), so no count
   ever triggers a collective allocation;
2. layout (identical on all ranks, from the matrix): for the owner ``d`` of
   expert ``e = d*El + j`` the rows of expert ``j`` start at a multiple of 128
   and are ordered by source rank; row ``k`` of source ``s`` for expert ``e``
   lands at ``pstart[d, j] + sum_{s'<s} M[s', e] + k``;
3. dispatch = ``ep_scatter_rows`` (P2P stores) bracketed by epoch barriers;
   padding rows are zeroed; the grouped SwiGLU runs on the padded buffer;
4. combine = outputs copied into the symmetric buffer, barrier,
   ``ep_gather_rows`` (P2P loads) into token order, barrier.

Backward mirrors it: dispatch backward is a gather of the input gradients at
the same positions, combine backward a scatter of the output gradients.

On CPU (gloo) the same plan runs with ``comm="collective"``: all-to-alls
emulate the peer stores and loads exactly (tests compare it with the NCCL path).
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist
import torch.nn as nn

TILE = 128


class Plan:
    """Per-call layout. ``dest_rank`` / ``dest_row`` (where each of my routed rows goes) are
    computed on the device from the count matrix, so the dispatch can be launched before the
    host has seen the counts; ``finalize`` adds the host-side sizes (padded rows received here)
    once the matrix's copy to pinned host memory has landed."""

    def __init__(self, M: torch.Tensor, me: int, device: torch.device, n_rows: int | None = None):
        M = M.to(device)
        ep, E = M.shape
        El = E // ep
        n_rows = int(M[me].sum()) if n_rows is None else n_rows
        T = M.sum(0).view(ep, El)                       # rows per (owner, local expert)
        pad = (T + TILE - 1) // TILE * TILE
        pstart = torch.cumsum(pad, 1) - pad             # [ep, El]
        before = torch.cumsum(M, 0) - M                 # rows of earlier sources, per expert [ep, E]
        off = pstart.reshape(-1)[None, :] + before      # [ep(src), E] first row of (src, e)
        mine = M[me]                                     # my rows per global expert
        e_of_row = torch.repeat_interleave(torch.arange(E, device=device), mine, output_size=n_rows)
        first_of_e = torch.cumsum(mine, 0) - mine
        k = torch.arange(n_rows, device=device) - first_of_e[e_of_row]
        self.dest_rank = (e_of_row // El).to(torch.int32)
        self.dest_row = (off[me][e_of_row] + k).to(torch.int64)
        self.local_counts = T[me]                        # rows of each of my experts (device)
        self.me, self.El, self.device = me, El, device
        self.scattered = False  # set when the row stores were queued before finalize

    def finalize(self, M_host: torch.Tensor) -> "Plan":
        ep, E = M_host.shape
        T = M_host.sum(0).view(ep, self.El)
        pad = (T + TILE - 1) // TILE * TILE
        pstart = torch.cumsum(pad, 1) - pad
        me = self.me
        self.P = int(pad[me].sum())                      # padded rows I receive
        self.P_max = int(pad.sum(1).max())               # largest receive buffer over ranks
        real = torch.zeros(self.P, dtype=torch.bool)
        for j in range(self.El):
            s0 = int(pstart[me, j])
            real[s0:s0 + int(T[me, j])] = True
        self.pad_rows = (~real).nonzero().flatten().to(self.device, non_blocking=True)
        self.real_rows = real.nonzero().flatten().to(self.device, non_blocking=True)
        return self


class EPPeerComm:
    def __init__(self, group, num_experts: int, comm: str | None = None):
        self.group = group
        self.ep = dist.get_world_size(group)
        self.me = dist.get_rank(group)
        self.E = num_experts
        self.comm = comm
        self.cap = 0
        self.dim = 0
        self._epoch = 0
        self.last_max_rows = 0  # largest routed rows of one rank seen in a count matrix

    # ---------------------------------------------------------------- buffers
    def _symm(self):
        os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")  # plain peer loads/stores only
        from torch.distributed import _symmetric_memory as symm

        return symm

    def _setup_counts(self, device: torch.device) -> None:
        if self.comm is None:
            self.comm = "peer" if device.type == "cuda" else "collective"
        if self.comm != "peer" or hasattr(self, "cnt"):
            return
        from torchtitan_b200.ops._ext import ext

        symm, name = self._symm(), self.group.group_name
        self._ext = ext()
        cols = -(-2 * self.E // 8) * 8  # int32 counts viewed as pairs of bf16: rows of 16-byte vectors
        self.cnt = symm.empty(self.ep, cols, dtype=torch.bfloat16, device=device)
        self.flags = symm.empty(self.ep, dtype=torch.int32, device=device)
        self.flags.zero_()
        self.cnt_ptrs = [int(x) for x in symm.rendezvous(self.cnt, name).buffer_ptrs]
        self.f_ptrs = [int(x) for x in symm.rendezvous(self.flags, name).buffer_ptrs]
        torch.cuda.synchronize(device)
        dist.barrier(group=self.group)

    def _ensure_rows(self, device: torch.device, dim: int, rows: int) -> None:
        """Grow the symmetric row buffers; every rank computes the same ``rows`` from the
        same count matrix, so the collective allocation happens on all ranks together."""
        if rows <= self.cap and dim == self.dim:
            return
        symm, name = self._symm(), self.group.group_name
        cap = max(rows, 2 * self.cap if dim == self.dim else 0, TILE)
        self.buf_in = symm.empty(cap, dim, dtype=torch.bfloat16, device=device)
        self.buf_out = symm.empty(cap, dim, dtype=torch.bfloat16, device=device)
        self.in_ptrs = [int(x) for x in symm.rendezvous(self.buf_in, name).buffer_ptrs]
        self.out_ptrs = [int(x) for x in symm.rendezvous(self.buf_out, name).buffer_ptrs]
        self.cap, self.dim = cap, dim
        torch.cuda.synchronize(device)
        dist.barrier(group=self.group)

    def bound(self, max_routed_rows: int) -> int:
        """Receive rows that cover any routing of ``max_routed_rows`` rows per source: all of
        them on one owner, plus one partial tile per local expert."""
        return self.ep * max_routed_rows + (self.E // self.ep) * TILE

    def reserve(self, device: torch.device, dim: int, max_routed_rows: int) -> None:
        """Size the receive buffers for the worst case of ``max_routed_rows`` (a value every
        rank holds: it comes from a count matrix all ranks share). The allocation is
        collective, so it happens when the largest per-rank batch grows, never per call."""
        if self.comm == "peer":
            self._ensure_rows(device, dim, self.bound(max_routed_rows))

    def barrier(self) -> None:
        if self.comm == "peer":
            self._epoch += 1
            self._ext.dp_barrier(self.f_ptrs, self.me, 0, self._epoch,
                                 limit_s=float(os.environ.get("TTB_DP_WAIT_S", "20")))
        else:
            dist.barrier(group=self.group)

    # ---------------------------------------------------------------- operations
    def exchange_counts(self, counts: torch.Tensor):
        """[E] routed rows per global expert on this rank -> ([ep, E] int64 on the device,
        the same matrix in host memory: a CPU tensor (collective mode) or, on CUDA, a pinned
        tensor filled by an asynchronous copy and the event that marks its completion)."""
        self._setup_counts(counts.device)
        if self.comm == "collective":
            out = [torch.empty_like(counts) for _ in range(self.ep)]
            dist.all_gather(out, counts.contiguous(), group=self.group)
            m = torch.stack(out).to(torch.int64).cpu()
            return m, m, None
        row = torch.zeros(self.cnt.shape[1] // 2, dtype=torch.int32, device=counts.device)
        row[:self.E] = counts.to(torch.int32)
        src = row.view(torch.bfloat16)[None].expand(self.ep, -1).contiguous()
        self.barrier()  # every peer is done reading its matrix from the previous call
        self._ext.ep_scatter_rows(src, torch.arange(self.ep, dtype=torch.int32, device=counts.device),
                                  torch.full((self.ep,), self.me, dtype=torch.int64, device=counts.device),
                                  self.cnt_ptrs, self.ep)
        self.barrier()
        m_dev = self.cnt.view(torch.int32)[:, :self.E].to(torch.int64)
        m_host = torch.empty(m_dev.shape, dtype=torch.int64, pin_memory=True)
        m_host.copy_(m_dev, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        return m_dev, m_host, ev

    def scatter(self, rows: torch.Tensor, dest_rank: torch.Tensor, dest_row: torch.Tensor, P: int,
                P_max: int) -> torch.Tensor:
        """Row i of ``rows`` -> row ``dest_row[i]`` of rank ``dest_rank[i]``; returns this rank's
        first ``P`` rows (rows nobody wrote are unspecified)."""
        if self.comm == "collective":
            send = [rows[dest_rank == r] for r in range(self.ep)]
            idx = [dest_row[dest_rank == r] for r in range(self.ep)]
            recv = _a2a_var(send, self.group)
            ridx = _a2a_var(idx, self.group)
            out = rows.new_zeros(P, rows.shape[1])
            out[ridx] = recv
            return out
        self.launch_scatter(rows, dest_rank, dest_row, P_max)
        return self.buf_in[:P].clone()

    def launch_scatter(self, rows: torch.Tensor, dest_rank: torch.Tensor, dest_row: torch.Tensor,
                       P_max: int | None = None) -> None:
        """Peer mode: queue the row stores and their barriers (no host information needed
        beyond the reserved capacity; ``ep_scatter_rows`` checks every row against it)."""
        if P_max is not None:
            self._ensure_rows(rows.device, rows.shape[1], P_max)
        self.barrier()  # peers are done with this buffer's previous contents
        self._ext.ep_scatter_rows(rows.contiguous(), dest_rank, dest_row, self.in_ptrs, self.cap)
        self.barrier()  # every peer's rows have landed here

    def gather(self, local: torch.Tensor, src_rank: torch.Tensor, src_row: torch.Tensor, P_max: int) -> torch.Tensor:
        """Expose ``local`` [P, D]; return rows ``src_row[i]`` of rank ``src_rank[i]``'s exposed rows."""
        if self.comm == "collective":
            want = [src_row[src_rank == r] for r in range(self.ep)]
            asked, sizes = _a2a_var(want, self.group, return_sizes=True)
            reply = list(local[asked].split(sizes))
            got = _a2a_var(reply, self.group).split([t.shape[0] for t in want])
            out = local.new_empty(src_row.shape[0], local.shape[1])
            for r in range(self.ep):
                out[src_rank == r] = got[r]
            return out
        self._ensure_rows(local.device, local.shape[1], P_max)
        self.barrier()  # peers are done reading this buffer's previous contents
        self.buf_out[:local.shape[0]].copy_(local)
        self.barrier()  # every peer's outputs are exposed
        out = local.new_empty(src_row.shape[0], local.shape[1])
        self._ext.ep_gather_rows(out, src_rank, src_row, self.out_ptrs, self.cap)
        return out


def _a2a_var(chunks: list[torch.Tensor], group, return_sizes: bool = False):
    """All-to-all of variable-length chunks (chunk r goes to rank r); returns the
    concatenation of what every rank sent here (and the per-source lengths)."""
    sizes = torch.tensor([c.shape[0] for c in chunks], dtype=torch.int64)
    in_sizes = torch.empty_like(sizes)
    dist.all_to_all_single(in_sizes, sizes, group=group)
    send = torch.cat(chunks)
    recv = send.new_empty((int(in_sizes.sum()),) + tuple(send.shape[1:]))
    dist.all_to_all_single(recv, send, in_sizes.tolist(), sizes.tolist(), group=group)
    return (recv, in_sizes.tolist()) if return_sizes else recv


class _Dispatch(torch.autograd.Function):
    @staticmethod
    def forward(ctx, routed, comm: EPPeerComm, plan: Plan):
        ctx.comm, ctx.plan = comm, plan
        if plan.scattered:  # the stores were queued before the host saw the counts
            xp = comm.buf_in[:plan.P].clone()
        else:
            xp = comm.scatter(routed, plan.dest_rank, plan.dest_row, plan.P, plan.P_max)
        if plan.pad_rows.numel():
            xp[plan.pad_rows] = 0
        return xp

    @staticmethod
    def backward(ctx, gxp):
        p = ctx.plan
        return ctx.comm.gather(gxp.contiguous(), p.dest_rank, p.dest_row, p.P_max), None, None


class _Combine(torch.autograd.Function):
    @staticmethod
    def forward(ctx, yp, comm: EPPeerComm, plan: Plan):
        ctx.comm, ctx.plan = comm, plan
        return comm.gather(yp.contiguous(), plan.dest_rank, plan.dest_row, plan.P_max)

    @staticmethod
    def backward(ctx, gout):
        p = ctx.plan
        gyp = ctx.comm.scatter(gout.contiguous(), p.dest_rank, p.dest_row, p.P, p.P_max)
        if p.pad_rows.numel():
            gyp[p.pad_rows] = 0
        return gyp, None, None


def make_fused_ep_dispatch(ep_group, num_experts: int, comm: str | None = None):
    """Drop-in for ``expert_parallel.make_ep_dispatch``: ``dispatch(routed, counts, experts)``
    with ``routed`` sorted by global expert and ``counts`` [E] per expert."""
    ep = dist.get_world_size(ep_group)
    if num_experts % ep:
        raise ValueError(f"num_experts {num_experts} not divisible by ep degree {ep}")
    pc = EPPeerComm(ep_group, num_experts, comm)

    def dispatch(routed: torch.Tensor, counts: torch.Tensor, experts: nn.Module) -> torch.Tensor:
        from torchtitan_b200 import ops
        from torchtitan_b200.models.common.moe import GroupedExperts

        m_dev, m_host, ev = pc.exchange_counts(counts)  # (decides the comm mode on first use)
        if pc.comm == "peer" and routed.dtype != torch.bfloat16:
            routed = routed.to(torch.bfloat16)
        plan = Plan(m_dev, pc.me, routed.device, n_rows=routed.shape[0])
        # decided from what every rank shares (the reserved size and earlier count matrices), so
        # all ranks take the same branch and issue the same barriers
        early = (pc.comm == "peer" and pc.dim == routed.shape[1] and pc.last_max_rows > 0
                 and pc.cap >= pc.bound(pc.last_max_rows))
        if early:
            # the row stores go out while the count matrix travels to the host; they are
            # bounds-checked against the reserved rows
            pc.launch_scatter(routed.contiguous(), plan.dest_rank, plan.dest_row)
            plan.scattered = True
        if ev is not None:
            ev.synchronize()
        plan.finalize(m_host)
        if pc.comm == "peer":
            rows_per_rank = m_host.sum(1)
            pc.last_max_rows = max(pc.last_max_rows, int(rows_per_rank.max()))
            if early and plan.P_max > pc.cap:
                # more rows than any earlier call: rows past the reserved buffer were skipped
                # (and flagged); every rank sees the same matrix, grows and stores again
                torch.cuda.synchronize(routed.device)
                pc._ext.ep_error_code(True)
                plan.scattered = False
            if not plan.scattered:
                pc.reserve(routed.device, routed.shape[1], pc.last_max_rows)
        xp = _Dispatch.apply(routed.contiguous(), pc, plan)
        if type(experts) is GroupedExperts:
            yp = ops.grouped_swiglu_padded(xp, *experts.weights(), plan.local_counts)
        else:  # any other expert module sees its rows unpadded
            y = experts(xp[plan.real_rows], plan.local_counts)
            yp = y.new_zeros(plan.P, y.shape[1]).index_copy(0, plan.real_rows, y)
        return _Combine.apply(yp.to(routed.dtype), pc, plan)

    dispatch.comm = pc
    return dispatch
