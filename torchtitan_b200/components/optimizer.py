"""Optimizers: fused AdamW, Muon and DistMuon, wrapped in a DCP-friendly container.

Parity: ``torchtitan/components/optimizer.py:38-444`` (container, regex param
groups, flattened DCP state, MoE bias pre-hook).  Beyond the reference:
``Muon`` / ``DistMuon`` (the reference has only Adam/AdamW).

* ``AdamW`` with ``implementation="fused"`` runs ``ops.fused_adamw_`` -- one
  multi-tensor sm_100a kernel over every local shard (fp32 master, fp32
  moments) per step.
* ``Muon`` applies Newton-Schulz orthogonalised momentum to 2-D hidden
  matrices (Jordan et al. 2024, "Muon: an optimizer for hidden layers",
  quintic iteration with coefficients (3.4445, -4.7750, 2.0315)) and AdamW to
  everything else (embeddings, output head, norms, biases, 1-D params).
* ``DistMuon`` is Muon for sharded (DTensor) parameters: each matrix is
  assigned an owner rank round-robin; shards are gathered to the owner, the
  owner orthogonalises, and the update is scattered back as shards.
"""
from __future__ import annotations

import functools
import re
from collections import defaultdict
from dataclasses import dataclass, field
from typing import Any, Literal

import torch
import torch.distributed as dist
import torch.nn as nn
from torch.distributed.checkpoint.state_dict import (
    StateDictOptions,
    get_optimizer_state_dict,
    set_optimizer_state_dict,
)
from torch.distributed.checkpoint.stateful import Stateful

from torchtitan_b200 import ops
from torchtitan_b200.config import Configurable
from torchtitan_b200.utils.logging import logger

try:
    from torch.distributed.tensor import DTensor, Shard
except ImportError:  # pragma: no cover
    DTensor = ()  # type: ignore


def _local(t: torch.Tensor) -> torch.Tensor:
    return t.to_local() if isinstance(t, DTensor) else t


def _load_keeping_fp32(opt: torch.optim.Optimizer, state_dict) -> None:
    """torch casts loaded state to each parameter's dtype; master-backed
    parameters are bf16 compute weights, so they are pointed at their fp32
    masters while loading, then the masters restored from the state drive them."""
    swapped = []
    for group in opt.param_groups:
        for p in group["params"]:
            if hasattr(p, "_master") and p.dtype != p._master.dtype:
                swapped.append((p, p.data))
                p.data = p._master
    try:
        torch.optim.Optimizer.load_state_dict(opt, state_dict)
    finally:
        with torch.no_grad():
            for p, compute in swapped:
                m = opt.state.get(p, {}).get("master")
                if m is not None:
                    p._master.copy_(m)
                    opt.state[p]["master"] = p._master
                compute.copy_(p._master)
                p.data = compute


class AdamW(torch.optim.Optimizer):
    """AdamW with decoupled weight decay.  ``fused=True`` on CUDA runs one
    multi-tensor kernel per (dtype, device) group and step."""

    def __init__(self, params, lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.0, fused=True):
        super().__init__(params, dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay, fused=fused))
        self.pending_clip: tuple[torch.Tensor, float] | None = None  # (sum of squares, max_norm) for the next step

    supports_fused_clip = True

    @torch.no_grad()
    def step(self, closure=None):
        loss = closure() if closure is not None else None
        for group in self.param_groups:
            ps, gs, ms, vs, steps, copies = [], [], [], [], [], []
            for p in group["params"]:
                if p.grad is None:
                    continue
                st = self.state[p]
                master = getattr(p, "_master", None)
                if not st:
                    st["step"] = torch.zeros((), dtype=torch.float32)
                    ref = master if master is not None else p
                    st["exp_avg"] = torch.zeros_like(ref, memory_format=torch.preserve_format)
                    st["exp_avg_sq"] = torch.zeros_like(ref, memory_format=torch.preserve_format)
                    if master is not None:
                        st["master"] = master  # saved with the optimizer state
                st["step"] += 1
                if master is not None:
                    ps.append(master); copies.append(p.data)
                else:
                    ps.append(_local(p)); copies.append(None)
                gs.append(_local(p.grad))
                ms.append(_local(st["exp_avg"])); vs.append(_local(st["exp_avg_sq"]))
                steps.append(int(st["step"].item()))
            if not ps:
                continue
            b1, b2 = group["betas"]
            lr = group["lr"]
            lr = float(lr.item()) if torch.is_tensor(lr) else float(lr)
            # all params of a group advance together, so a single step count is used
            clip_total, clip_max = self.pending_clip if self.pending_clip is not None else (None, 0.0)
            ops.fused_adamw_(ps, gs, ms, vs, lr=lr, beta1=b1, beta2=b2, eps=group["eps"],
                             weight_decay=group["weight_decay"], step=steps[0],
                             copies=copies if any(c is not None for c in copies) else None,
                             clip_total=clip_total, clip_max=clip_max)
        self.pending_clip = None
        return loss

    def load_state_dict(self, state_dict):
        _load_keeping_fp32(self, state_dict)
        for g in self.param_groups:  # re-read the step count from the loaded state on next use
            g.pop("_host_step", None)


class PeerShardedAdamW(torch.optim.Optimizer):
    """AdamW over the sharded fp32 state of a :class:`PeerDataParallel` runtime.

    ``param_groups`` list the model's parameters (so LR schedulers work as
    usual); the state is three flat fp32 shards (master, exp_avg, exp_avg_sq)
    covering this rank's 1/W slice of every gradient bucket.  One fused kernel
    updates them and writes the new bf16 weights into every rank's buffer."""

    supports_fused_clip = True

    def __init__(self, groups, runtime):
        super().__init__(groups, {})
        keys = ("lr", "betas", "eps", "weight_decay")
        g0 = self.param_groups[0]
        for g in self.param_groups[1:]:
            if any(g[k] != g0[k] for k in keys):
                raise ValueError("peer data parallelism runs one AdamW hyper-parameter set over the flat shard; "
                                 "use data_parallel_comm='fsdp2' for per-group settings")
        self.rt = runtime
        self.exp_avg = torch.zeros_like(runtime.master)
        self.exp_avg_sq = torch.zeros_like(runtime.master)
        self.step_count = 0
        self.pending_clip: tuple[torch.Tensor, float] | None = None

    @torch.no_grad()
    def step(self, closure=None):
        loss = closure() if closure is not None else None
        g = self.param_groups[0]
        lr = float(g["lr"].item()) if torch.is_tensor(g["lr"]) else float(g["lr"])
        self.step_count += 1
        self.rt.adamw_step(self.exp_avg, self.exp_avg_sq, lr=lr, beta1=g["betas"][0], beta2=g["betas"][1],
                           eps=g["eps"], weight_decay=g["weight_decay"], step=self.step_count, clip=self.pending_clip)
        self.pending_clip = None
        return loss

    def zero_grad(self, set_to_none: bool = True):
        pass  # gradients never stay on the parameters: the runtime's hooks move them into its buffers

    def _dtensor(self, t: torch.Tensor):
        from torch.distributed.tensor import DTensor, Shard

        return DTensor.from_local(t.view(1, -1), self.rt.flat_mesh, [Shard(0)], run_check=False)

    def flat_state_dict(self) -> dict[str, Any]:
        return {"peer_dp.master": self._dtensor(self.rt.master), "peer_dp.exp_avg": self._dtensor(self.exp_avg),
                "peer_dp.exp_avg_sq": self._dtensor(self.exp_avg_sq),
                "peer_dp.step": torch.tensor(self.step_count, dtype=torch.int64),
                # the LR scheduler restores its counter only; the current lr lives in the groups
                "peer_dp.lr": torch.tensor([float(g["lr"]) for g in self.param_groups], dtype=torch.float64)}

    @torch.no_grad()
    def load_flat_state_dict(self, sd: dict[str, Any]) -> None:
        for key, t in (("master", self.rt.master), ("exp_avg", self.exp_avg), ("exp_avg_sq", self.exp_avg_sq)):
            v = sd[f"peer_dp.{key}"]
            v = v.to_local() if hasattr(v, "to_local") else v
            if v.data_ptr() != t.data_ptr():
                t.copy_(v.reshape(-1))
        self.step_count = int(sd["peer_dp.step"])
        if "peer_dp.lr" in sd:
            for g, lr in zip(self.param_groups, sd["peer_dp.lr"].tolist()):
                g["lr"] = lr
        self.rt.gather_weights()


def zeropower_via_newtonschulz5(G: torch.Tensor, steps: int = 5, eps: float = 1e-7) -> torch.Tensor:
    """Approximate the orthogonal polar factor of ``G`` (Muon's quintic
    Newton-Schulz iteration, coefficients from Jordan et al. 2024)."""
    a, b, c = 3.4445, -4.7750, 2.0315
    X = G.to(torch.bfloat16 if G.is_cuda else torch.float32)
    transposed = X.size(-2) > X.size(-1)
    if transposed:
        X = X.mT
    X = X / (X.norm(dim=(-2, -1), keepdim=True) + eps)
    for _ in range(steps):
        A = ops.matmul(X, X.mT)
        B = b * A + c * ops.matmul(A, A)
        X = a * X + ops.matmul(B, X)
    if transposed:
        X = X.mT
    return X.to(G.dtype)


def _muon_scale(shape: torch.Size) -> float:
    # match AdamW update RMS (Moonshot "Muon is scalable", 0.2*sqrt(max(m,n)))
    return 0.2 * max(shape[-2], shape[-1]) ** 0.5


class Muon(torch.optim.Optimizer):
    """Muon for 2-D ``muon`` groups, AdamW (fused kernel) for the rest.

    Param groups carry ``use_muon``.  Parameters may be DTensors: in that
    case ``distributed=True`` (DistMuon) gathers each matrix to an owner rank.
    """

    def __init__(self, params, lr=0.02, momentum=0.95, nesterov=True, ns_steps=5, betas=(0.9, 0.95),
                 eps=1e-8, weight_decay=0.0, distributed=False):
        super().__init__(params, dict(lr=lr, momentum=momentum, nesterov=nesterov, ns_steps=ns_steps,
                                      betas=betas, eps=eps, weight_decay=weight_decay, use_muon=True))
        self.distributed = distributed

    def load_state_dict(self, state_dict):
        _load_keeping_fp32(self, state_dict)

    def _orthogonalize_all(self, items: list[tuple[torch.Tensor, torch.Tensor]], ns_steps: int) -> list[torch.Tensor]:
        """``items``: (param, momentum-update) pairs; returns per-param local updates."""
        if not self.distributed or not any(isinstance(u, DTensor) for _, u in items):
            return [zeropower_via_newtonschulz5(_full(u), ns_steps) for _, u in items]
        out: list[torch.Tensor | None] = [None] * len(items)
        by_group: dict[Any, list[tuple[int, DTensor]]] = {}
        for idx, (_, u) in enumerate(items):
            if not isinstance(u, DTensor):
                out[idx] = zeropower_via_newtonschulz5(u, ns_steps)
                continue
            shard_dims = [i for i, pl in enumerate(u.placements) if isinstance(pl, Shard)]
            if len(shard_dims) == 1 and u.placements[shard_dims[0]].dim == 0:
                by_group.setdefault(u.device_mesh.get_group(shard_dims[0]), []).append((idx, u))
            else:
                out[idx] = _dist_orthogonalize(u, idx, ns_steps)
        for pg, lst in by_group.items():
            for idx, res in _dist_orthogonalize_bucketed(pg, lst, ns_steps).items():
                out[idx] = res
        return out  # type: ignore

    @torch.no_grad()
    def step(self, closure=None):
        loss = closure() if closure is not None else None
        for group in self.param_groups:
            params = [p for p in group["params"] if p.grad is not None]
            if not params:
                continue
            lr, wd = float(group["lr"]), group["weight_decay"]
            if not group["use_muon"]:
                ps, gs, ms, vs = [], [], [], []
                copies = []
                for p in params:
                    st = self.state[p]
                    master = getattr(p, "_master", None)
                    ref = master if master is not None else p
                    if not st:
                        st["step"] = torch.zeros(())
                        st["exp_avg"] = torch.zeros_like(ref)
                        st["exp_avg_sq"] = torch.zeros_like(ref)
                    st["step"] += 1
                    ps.append(master if master is not None else _local(p))
                    copies.append(p.data if master is not None else None)
                    gs.append(_local(p.grad))
                    ms.append(_local(st["exp_avg"])); vs.append(_local(st["exp_avg_sq"]))
                b1, b2 = group["betas"]
                # the step count is mirrored on the host so the kernel launch needs no device sync
                host_step = group.get("_host_step")
                if host_step is None:
                    host_step = int(self.state[params[0]]["step"].item())
                else:
                    host_step += 1
                group["_host_step"] = host_step
                ops.fused_adamw_(ps, gs, ms, vs, lr=lr, beta1=b1, beta2=b2, eps=group["eps"], weight_decay=wd,
                                 step=host_step,
                                 copies=copies if any(c is not None for c in copies) else None)
                continue
            mom = group["momentum"]
            items = []
            for p in params:
                st = self.state[p]
                if "momentum_buffer" not in st:
                    st["momentum_buffer"] = torch.zeros_like(getattr(p, "_master", p))
                buf = st["momentum_buffer"]
                grad = p.grad.to(buf.dtype)
                buf.mul_(mom).add_(grad)
                upd = grad.add(buf, alpha=mom) if group["nesterov"] else buf
                items.append((p, upd))
            updates = self._orthogonalize_all(items, group["ns_steps"])
            for (p, _), u in zip(items, updates):
                master = getattr(p, "_master", None)
                pl = master if master is not None else _local(p)
                if wd:
                    pl.mul_(1 - lr * wd)
                pl.add_(u.to(pl.dtype), alpha=-lr * _muon_scale(p.shape))
                if master is not None:
                    p.data.copy_(master)
        return loss


def _full(t: torch.Tensor) -> torch.Tensor:
    return t.full_tensor() if isinstance(t, DTensor) else t


def _ns_batched(mats: list[torch.Tensor], ns_steps: int) -> list[torch.Tensor]:
    """Newton-Schulz on many matrices: equal trailing shapes are stacked and iterated together
    (on CUDA each iteration's products are single grouped GEMMs over the whole stack)."""
    out: list[torch.Tensor | None] = [None] * len(mats)
    by_shape: dict[tuple[int, int], list[int]] = {}
    for i, m in enumerate(mats):
        by_shape.setdefault(tuple(m.shape[-2:]), []).append(i)
    for shape, ids in by_shape.items():
        stack = torch.cat([mats[i].reshape(-1, *shape) for i in ids])
        res = zeropower_via_newtonschulz5(stack, ns_steps)
        pos = 0
        for i in ids:
            n = mats[i].numel() // (shape[0] * shape[1])
            out[i] = res[pos:pos + n].reshape(mats[i].shape)
            pos += n
    return out  # type: ignore


def _dist_orthogonalize_bucketed(pg, lst: list[tuple[int, "DTensor"]], ns_steps: int,
                                 waves: int = 2) -> dict[int, torch.Tensor]:
    """DistMuon over one process group for every Shard(0) matrix at once.

    Owners are assigned greedily by size (largest first, to the least-loaded rank), so every
    rank orthogonalises its share concurrently. One all-to-all carries every rank's row chunk of
    every matrix to its owner, the owner runs batched Newton-Schulz on all of its matrices, and
    a second all-to-all returns the row chunks: two collectives per wave, not two per parameter.
    The matrices are split into ``waves`` size-balanced waves that are pipelined: the
    all-to-all bringing wave w+1 to its owners and the one returning wave w-1 run (asynchronously,
    on the communicator's stream) while wave w is orthogonalised.
    (The reference has no distributed Muon: its optimizer registry stops at AdamW/Adam,
    ``torchtitan/components/optimizer.py:130-134``.)
    """
    world, rank = dist.get_world_size(pg), dist.get_rank(pg)
    dev = lst[0][1].to_local().device
    wire = torch.bfloat16 if dev.type == "cuda" else torch.float32  # NS runs in bf16 on CUDA
    order = sorted(range(len(lst)), key=lambda j: -lst[j][1].numel())
    load = [0] * world
    owner = [0] * len(lst)
    for j in order:
        o = min(range(world), key=lambda r: load[r])
        owner[j] = o
        load[o] += lst[j][1].numel()
    rows = [u.shape[0] for _, u in lst]
    inner = [u.numel() // max(u.shape[0], 1) for _, u in lst]
    chunk = [(r + world - 1) // world for r in rows]
    cnum = [c * i for c, i in zip(chunk, inner)]
    # waves: the size order dealt round-robin, so every wave carries a similar share
    nw = max(1, min(waves, len(lst)))
    wave_of = {j: k % nw for k, j in enumerate(order)}

    def start_gather(w: int):
        js = [j for j in range(len(lst)) if wave_of[j] == w]
        mine = [j for j in js if owner[j] == rank]
        send = []
        for dst in range(world):
            for j in js:
                if owner[j] != dst:
                    continue
                loc = lst[j][1].to_local().reshape(-1, inner[j]).to(wire)
                buf = torch.zeros(chunk[j], inner[j], dtype=wire, device=dev)
                buf[:loc.shape[0]].copy_(loc)
                send.append(buf.reshape(-1))
        in_splits = [sum(cnum[j] for j in js if owner[j] == dst) for dst in range(world)]
        out_splits = [sum(cnum[j] for j in mine)] * world
        send_t = torch.cat(send) if send else torch.zeros(0, dtype=wire, device=dev)
        recv = torch.empty(sum(out_splits), dtype=wire, device=dev)
        work = dist.all_to_all_single(recv, send_t, out_splits, in_splits, group=pg, async_op=True)
        return js, mine, in_splits, out_splits, recv, send_t, work

    def orthogonalise(state):
        js, mine, in_splits, out_splits, recv, _send, work = state
        work.wait()
        per_src = recv.split(out_splits) if out_splits[0] else [recv] * world
        fulls = []
        for k, j in enumerate(mine):
            off = sum(cnum[jj] for jj in mine[:k])
            parts = [per_src[src][off:off + cnum[j]].view(chunk[j], inner[j]) for src in range(world)]
            fulls.append(torch.cat(parts)[:rows[j]].reshape(lst[j][1].shape))
        results = _ns_batched(fulls, ns_steps) if fulls else []
        back = []
        for dst in range(world):
            for k, j in enumerate(mine):
                r2 = results[k].reshape(rows[j], inner[j])
                buf = torch.zeros(chunk[j], inner[j], dtype=wire, device=dev)
                seg = r2[dst * chunk[j]:(dst + 1) * chunk[j]]
                buf[:seg.shape[0]].copy_(seg)
                back.append(buf.reshape(-1))
        back_t = torch.cat(back) if back else torch.zeros(0, dtype=wire, device=dev)
        recv2 = torch.empty(sum(in_splits), dtype=wire, device=dev)
        work2 = dist.all_to_all_single(recv2, back_t, in_splits, out_splits, group=pg, async_op=True)
        return js, recv2, back_t, work2

    out: dict[int, torch.Tensor] = {}

    def finish(state):
        js, recv2, _back, work2 = state
        work2.wait()
        pos = 0  # this rank's rows of every matrix of the wave, in the order of the owners' sends
        for src in range(world):
            for j in js:
                if owner[j] != src:
                    continue
                loc = lst[j][1].to_local()
                piece = recv2[pos:pos + cnum[j]].view(chunk[j], inner[j])[:loc.shape[0]]
                out[lst[j][0]] = piece.reshape(loc.shape).to(loc.dtype)
                pos += cnum[j]

    pending = start_gather(0)
    returning = []
    for w in range(nw):
        nxt = start_gather(w + 1) if w + 1 < nw else None  # next wave in flight during this NS
        returning.append(orthogonalise(pending))
        pending = nxt
    for st in returning:
        finish(st)
    return out


def _dist_orthogonalize(u: "DTensor", idx: int, ns_steps: int) -> torch.Tensor:
    """Gather ``u``'s Shard(0) pieces to owner ``idx % world``, orthogonalise
    there, scatter the result back.  Other placements fall back to full_tensor."""
    mesh, pl = u.device_mesh, u.placements
    shard_dims = [i for i, p in enumerate(pl) if isinstance(p, Shard)]
    if len(shard_dims) != 1 or pl[shard_dims[0]].dim != 0:
        full = zeropower_via_newtonschulz5(u.full_tensor(), ns_steps)
        return DTensor.from_local(full, mesh, [torch.distributed.tensor.Replicate()] * mesh.ndim).redistribute(
            mesh, pl).to_local()
    group = mesh.get_group(shard_dims[0])
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    owner = idx % world
    owner_global = dist.get_global_rank(group, owner)
    local = u.to_local().contiguous()
    rows = u.shape[0]
    chunk = (rows + world - 1) // world
    pad = torch.zeros((chunk,) + tuple(u.shape[1:]), dtype=local.dtype, device=local.device)
    pad[: local.shape[0]].copy_(local)
    gathered = [torch.empty_like(pad) for _ in range(world)] if rank == owner else None
    dist.gather(pad, gathered, dst=owner_global, group=group)
    recv = torch.empty_like(pad)
    if rank == owner:
        full = torch.cat(gathered, 0)[:rows]
        o = zeropower_via_newtonschulz5(full, ns_steps)
        parts = list(torch.nn.functional.pad(o, (0, 0) * (o.dim() - 1) + (0, chunk * world - rows)).split(chunk, 0))
        parts = [p.contiguous() for p in parts]
    else:
        parts = None
    dist.scatter(recv, parts, src=owner_global, group=group)
    return recv[: local.shape[0]]


@dataclass(kw_only=True, slots=True)
class ParamGroupConfig:
    pattern: str = ""
    lr_multiplier: float = 1.0
    weight_decay_multiplier: float = 1.0


class OptimizersContainer(Stateful, Configurable):
    """One optimizer per model part; behaves like a single optimizer."""

    @dataclass(kw_only=True, slots=True)
    class Config(Configurable.Config):
        name: str = "AdamW"
        """AdamW | Adam | Muon | DistMuon"""
        lr: float = 8e-4
        beta1: float = 0.9
        beta2: float = 0.95
        eps: float = 1e-8
        weight_decay: float = 0.1
        implementation: Literal["for-loop", "foreach", "fused"] = "fused"
        param_groups: list[ParamGroupConfig] = field(default_factory=list)
        muon_lr: float = 0.02
        muon_momentum: float = 0.95
        muon_ns_steps: int = 5
        muon_exclude_patterns: list[str] = field(
            default_factory=lambda: ["tok_embeddings", "embed_tokens", "output", "lm_head", "norm", "router", "bias"]
        )
        early_step_in_backward: bool = False
        """Step each parameter inside backward, as soon as its gradient is accumulated, and free
        the gradient right away (the reference's ``OptimizersInBackwardContainer``): gradient
        memory drops to one parameter's worth; no gradient clipping, no gradient accumulation."""

    def __init__(self, config: Config, *, model_parts: list[nn.Module], **kw: Any):
        self.config = config
        self.model_parts = model_parts
        self.optimizers: list[torch.optim.Optimizer] = []
        self._pre_hooks: list[Any] = []
        self._post_hooks: list[Any] = []
        self._parts_of: list[nn.Module] = []  # model part of each optimizer (state-dict flattening)
        if config.early_step_in_backward:
            self._build_in_backward(model_parts)
            return
        for m in model_parts:
            self.optimizers.append(self._build_one(m))
            self._parts_of.append(m)

    def _build_in_backward(self, model_parts: list[nn.Module]) -> None:
        """One optimizer per parameter, stepped from its post-accumulate-grad hook
        (parity: ``components/optimizer.py:277-335`` of the reference)."""
        if self.config.name not in ("AdamW", "Adam"):
            raise NotImplementedError("early_step_in_backward supports AdamW/Adam")
        for m in model_parts:
            opt = self._build_one(m)
            for g in opt.param_groups:
                hp = {k: v for k, v in g.items() if k != "params"}
                for p in g["params"]:
                    single = type(opt)([{"params": [p], **hp}], **({"fused": True} if isinstance(opt, AdamW) else {}))
                    self.optimizers.append(single)
                    self._parts_of.append(m)

                    def hook(param, _o=single):
                        _o.step()
                        _o.zero_grad(set_to_none=True)

                    p.register_post_accumulate_grad_hook(hook)

    def _groups(self, model: nn.Module, base: dict[str, Any]) -> list[dict[str, Any]]:
        pats = [re.compile(pg.pattern) for pg in self.config.param_groups]
        buckets: dict[int | None, list[tuple[str, nn.Parameter]]] = defaultdict(list)
        for n, p in model.named_parameters():
            if not p.requires_grad:
                continue
            hit = next((i for i, r in enumerate(pats) if r.search(n)), None)
            buckets[hit].append((n, p))
        groups = []
        for key, items in buckets.items():
            kw = dict(base)
            if key is not None:
                pg = self.config.param_groups[key]
                kw["lr"] = base["lr"] * pg.lr_multiplier
                kw["weight_decay"] = base["weight_decay"] * pg.weight_decay_multiplier
            groups.append({"params": items, **kw})
        for i, pg in enumerate(self.config.param_groups):
            if i not in buckets:
                logger.warning(f"optimizer param_groups pattern '{pg.pattern}' matched nothing")
        return groups

    def _build_one(self, model: nn.Module) -> torch.optim.Optimizer:
        c = self.config
        base = dict(lr=c.lr, betas=(c.beta1, c.beta2), eps=c.eps, weight_decay=c.weight_decay)
        groups = self._groups(model, base)
        rt = getattr(model, "_dp_runtime", None)
        if rt is not None:
            if c.name not in ("AdamW", "Adam"):
                raise NotImplementedError(f"peer data parallelism runs AdamW/Adam, not {c.name}; "
                                          "use data_parallel_comm='fsdp2'")
            for g in groups:
                g["params"] = [p for _, p in g["params"]]
                g["weight_decay"] *= 1.0 if c.name == "AdamW" else 0.0
            return PeerShardedAdamW(groups, rt)
        if c.name in ("AdamW", "Adam"):
            wd_scale = 1.0 if c.name == "AdamW" else 0.0
            for g in groups:
                g["params"] = [p for _, p in g["params"]]
                g["weight_decay"] *= wd_scale
            if c.implementation == "fused":
                return AdamW(groups, fused=True)
            return torch.optim.AdamW(groups, foreach=c.implementation == "foreach") if c.name == "AdamW" else \
                torch.optim.Adam(groups, foreach=c.implementation == "foreach")
        if c.name in ("Muon", "DistMuon"):
            excl = [re.compile(p) for p in c.muon_exclude_patterns]
            out = []
            for g in groups:
                mu = [p for n, p in g["params"] if p.ndim >= 2 and not any(r.search(n) for r in excl)]
                ad = [p for n, p in g["params"] if not (p.ndim >= 2 and not any(r.search(n) for r in excl))]
                rest = {k: v for k, v in g.items() if k != "params"}
                if mu:
                    out.append({"params": mu, **rest, "lr": c.muon_lr * rest["lr"] / c.lr, "use_muon": True})
                if ad:
                    out.append({"params": ad, **rest, "use_muon": False})
            return Muon(out, lr=c.muon_lr, momentum=c.muon_momentum, ns_steps=c.muon_ns_steps,
                        distributed=(c.name == "DistMuon"))
        raise NotImplementedError(f"optimizer {c.name}")

    # torch.optim.Optimizer-like surface ---------------------------------
    def __iter__(self):
        return iter(self.optimizers)

    def __len__(self):
        return len(self.optimizers)

    @property
    def param_groups(self):
        return [g for o in self.optimizers for g in o.param_groups]

    def register_step_pre_hook(self, hook) -> None:
        self._pre_hooks.append(hook)

    def register_step_post_hook(self, hook) -> None:
        self._post_hooks.append(hook)

    def step(self, *args, **kwargs) -> None:
        for h in self._pre_hooks:
            h(self, args, kwargs)
        if not self.config.early_step_in_backward:  # else every parameter already stepped in backward
            for o in self.optimizers:
                o.step(*args, **kwargs)
        for h in self._post_hooks:
            h(self, args, kwargs)

    def zero_grad(self, *args, **kwargs) -> None:
        for o in self.optimizers:
            o.zero_grad(set_to_none=True)

    def state_dict(self) -> dict[str, Any]:
        fn = functools.partial(get_optimizer_state_dict, options=StateDictOptions(flatten_optimizer_state_dict=True))
        out: dict[str, Any] = {}
        if self.config.early_step_in_backward:
            for m in self.model_parts:
                out.update(fn(m, [o for o, part in zip(self.optimizers, self._parts_of) if part is m]))
            return out
        for m, o in zip(self.model_parts, self.optimizers):
            out.update(o.flat_state_dict() if hasattr(o, "flat_state_dict") else fn(m, o))
        return out

    def load_state_dict(self, sd: dict[str, Any]) -> None:
        fn = functools.partial(set_optimizer_state_dict, optim_state_dict=sd,
                               options=StateDictOptions(flatten_optimizer_state_dict=True))
        if self.config.early_step_in_backward:
            for m in self.model_parts:
                fn(m, [o for o, part in zip(self.optimizers, self._parts_of) if part is m])
            return
        for m, o in zip(self.model_parts, self.optimizers):
            if hasattr(o, "load_flat_state_dict"):
                o.load_flat_state_dict(sd)
            else:
                fn(m, o)


def build_optimizers_with_moe_load_balancing(optimizers: OptimizersContainer, model_parts: list[nn.Module],
                                              parallel_dims: Any) -> None:
    """Register the aux-loss-free expert-bias update as a step pre-hook.

    Behaviour parity: ``torchtitan/components/optimizer.py:337-444``: the
    tokens-per-expert histogram of every MoE layer is summed across the loss
    mesh in one all-reduce, then ``bias += coeff * sign(mean - count)``
    (centred) and the histogram is cleared.
    """
    moes = [m for part in model_parts for m in part.modules() if getattr(m, "load_balance_coeff", None)]
    if not moes:
        return

    @torch.no_grad()
    def _update(*_a, **_k):
        counts = torch.stack([m.tokens_per_expert.float() for m in moes])
        mesh = parallel_dims.get_optional_mesh("loss") if parallel_dims is not None else None
        if mesh is not None:
            dist.all_reduce(counts, group=mesh.get_group())
        tp_group = getattr(moes[0], "tp_count_group", None)
        if tp_group is not None:  # sequence-parallel TP: each TP rank routed different tokens
            dist.all_reduce(counts, group=tp_group)
        for m, c in zip(moes, counts):
            delta = m.load_balance_coeff * torch.sign(c.mean() - c)
            m.expert_bias.add_(delta - delta.mean())
            m.tokens_per_expert.zero_()

    optimizers.register_step_pre_hook(_update)
