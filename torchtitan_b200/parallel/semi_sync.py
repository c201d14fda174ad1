"""Semi-synchronous data parallelism across replica groups: LocalSGD and
(streaming) DiLoCo (behaviour parity: reference ``experiments/ft/diloco/utils.py:15-136``,
``ft/manager.py:36-227``; the reference runs them through TorchFT, which is
not in this image).

The ``dp_replicate`` mesh dimension becomes a set of *replicas* that train
independently: gradients are reduced only inside a replica (FSDP over
``fsdp``), the loss is normalised by the replica's own token count, and every
``sync_steps`` steps the replicas synchronise their weights:

* ``local_sgd``: weights are averaged across replicas.
* ``diloco``: each replica keeps the weights of the last synchronisation
  (the *global* copy); the pseudo-gradient ``global - local`` is averaged
  across replicas and applied to the global copy by an outer SGD optimizer
  (Nesterov momentum by default, Douillard et al. 2023, "DiLoCo"); the
  replicas then restart from the new global weights (mixed with their own by
  ``fragment_update_alpha``).

With ``num_fragments > 1`` the model is cut into contiguous fragments whose
synchronisations are staggered evenly over the ``sync_steps`` window
("streaming DiLoCo", Douillard et al. 2025), so the communication is spread
out instead of arriving all at once.

Weights are synchronised on their local shards (every replica shards the same
way) and, for master-backed parameters, on the fp32 masters.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Literal

import torch
import torch.distributed as dist
import torch.nn as nn


@dataclass(kw_only=True, slots=True)
class FaultToleranceConfig:
    enable: bool = False
    semi_sync_method: Literal["local_sgd", "diloco"] | None = None
    sync_steps: int = 20
    num_fragments: int = 1
    fragment_update_alpha: float = 0.0
    """0 = restart from the new global weights; a > 0 keeps a fraction of the local ones."""
    outer_lr: float = 0.7
    outer_momentum: float = 0.9
    outer_nesterov: bool = True
    # dynamic replica groups (no semi_sync_method): each replica is its own job; replicas meet
    # at a lighthouse store and agree on a quorum every step (``parallel/ft.py``)
    lighthouse: str = ""
    """host:port of the lighthouse (``python -m torchtitan_b200.parallel.ft --port P``)."""
    replica_id: int = 0
    group_size: int = 0
    """Maximum number of replicas (data is sharded over ``group_size`` x the replica's DP degree)."""
    min_replica_size: int = 1
    quorum_timeout_s: float = 30.0
    process_group: Literal["gloo", "nccl"] = "gloo"
    process_group_timeout_ms: int = 10000


def _local(t: torch.Tensor) -> torch.Tensor:
    return t.to_local() if type(t).__name__ == "DTensor" else t


class SemiSync:
    def __init__(self, cfg: FaultToleranceConfig, model_parts: list[nn.Module], group):
        if cfg.semi_sync_method not in ("local_sgd", "diloco"):
            raise ValueError(f"unknown semi-sync method {cfg.semi_sync_method}")
        self.cfg, self.group = cfg, group
        self.n = dist.get_world_size(group)
        seen, params = set(), []
        for m in model_parts:
            for p in m.parameters():
                if p.requires_grad and id(p) not in seen:
                    seen.add(id(p))
                    params.append(p)
        k = max(1, min(cfg.num_fragments, len(params)))
        size = -(-len(params) // k)
        self.fragments = [params[i:i + size] for i in range(0, len(params), size)]
        self.offsets = [i * cfg.sync_steps // len(self.fragments) for i in range(len(self.fragments))]
        self.outer = []
        self.globals: list[list[torch.Tensor]] = []
        if cfg.semi_sync_method == "diloco":
            for frag in self.fragments:
                g = [self._weights(p).detach().clone() for p in frag]
                self.globals.append(g)
                self.outer.append(torch.optim.SGD(g, lr=cfg.outer_lr, momentum=cfg.outer_momentum,
                                                  nesterov=cfg.outer_nesterov and cfg.outer_momentum > 0))

    @staticmethod
    def _weights(p: torch.Tensor) -> torch.Tensor:
        """The tensor the optimizer owns: the fp32 master if there is one, else the local shard."""
        return getattr(p, "_master", None) if getattr(p, "_master", None) is not None else _local(p.data)

    @staticmethod
    def _push(p: torch.Tensor) -> None:
        m = getattr(p, "_master", None)
        if m is not None:
            p.data.copy_(m)

    def due(self, step: int) -> list[int]:
        return [i for i, off in enumerate(self.offsets) if step > 0 and (step - off) % self.cfg.sync_steps == 0
                and step >= self.cfg.sync_steps]

    @torch.no_grad()
    def after_step(self, step: int) -> list[int]:
        """Call after the optimizer step of ``step`` (1-based); returns the fragments synchronised."""
        idx = self.due(step)
        for i in idx:
            if self.cfg.semi_sync_method == "local_sgd":
                self._average(self.fragments[i])
            else:
                self._diloco(i)
        return idx

    def _average(self, frag: list[torch.Tensor]) -> None:
        ws = [self._weights(p) for p in frag]
        flat = torch.cat([w.reshape(-1).float() for w in ws])
        dist.all_reduce(flat, group=self.group)
        flat /= self.n
        o = 0
        for p, w in zip(frag, ws):
            w.copy_(flat[o:o + w.numel()].view_as(w))
            o += w.numel()
            self._push(p)

    def _diloco(self, i: int) -> None:
        frag, glob, opt = self.fragments[i], self.globals[i], self.outer[i]
        ws = [self._weights(p) for p in frag]
        pseudo = torch.cat([(g.float() - w.float()).reshape(-1) for g, w in zip(glob, ws)])
        dist.all_reduce(pseudo, group=self.group)
        pseudo /= self.n
        o = 0
        for g in glob:
            g.grad = pseudo[o:o + g.numel()].view_as(g).to(g.dtype)
            o += g.numel()
        opt.step()
        opt.zero_grad(set_to_none=True)
        a = self.cfg.fragment_update_alpha
        for p, g, w in zip(frag, glob, ws):
            w.copy_(g if a == 0 else a * w + (1 - a) * g)
            self._push(p)

    def state_dict(self) -> dict:
        if self.cfg.semi_sync_method != "diloco":
            return {}
        return {f"fragment_{i}": {"global": g, "outer": o.state_dict()}
                for i, (g, o) in enumerate(zip(self.globals, self.outer))}

    def load_state_dict(self, sd: dict) -> None:
        for i, (g, o) in enumerate(zip(self.globals, self.outer)):
            st = sd.get(f"fragment_{i}")
            if st:
                for dst, src in zip(g, st["global"]):
                    dst.copy_(src)
                o.load_state_dict(st["outer"])
