"""Parallel degrees and device meshes.

Dense ranks are laid out as ``[pp, dp_replicate, dp_shard, cp, tp]`` over
``arange(world)``; the MoE (sparse) layout re-splits the trailing
``dp_shard*cp*tp`` ranks as ``[efsdp, ep, etp]`` so an EP group is a set of
consecutive ranks (NVSwitch makes every peer equal on one node).  Named
meshes (parity: ``torchtitan/distributed/parallel_dims.py:22-397``):
``pp, dp_replicate, dp_shard, cp, tp`` plus flattened ``fsdp = dp_shard*cp``,
``batch = dp_replicate*dp_shard``, ``loss = batch*cp``, ``dp_cp``, and sparse
``efsdp, ep, etp``.  Meshes are created lazily; a degree-1 mesh is ``None``
from ``get_optional_mesh``.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any

import torch


@dataclass
class ParallelDims:
    dp_replicate: int
    dp_shard: int
    cp: int
    tp: int
    pp: int
    ep: int
    etp: int
    world_size: int
    _meshes: dict[str, Any] = field(default_factory=dict, repr=False)

    @classmethod
    def from_config(cls, p: Any, world_size: int) -> "ParallelDims":
        return cls(
            dp_replicate=p.data_parallel_replicate_degree,
            dp_shard=p.data_parallel_shard_degree,
            cp=p.context_parallel_degree,
            tp=p.tensor_parallel_degree,
            pp=p.pipeline_parallel_degree,
            ep=p.expert_parallel_degree,
            etp=p.expert_tensor_parallel_degree,
            world_size=world_size,
        )

    def __post_init__(self):
        for n in ("dp_replicate", "cp", "tp", "pp", "ep", "etp"):
            if getattr(self, n) < 1:
                raise ValueError(f"{n} degree must be >= 1")
        if self.dp_shard == -1:
            denom = self.dp_replicate * self.cp * self.tp * self.pp
            if self.world_size % denom:
                raise ValueError(f"world {self.world_size} not divisible by dp_replicate*cp*tp*pp={denom}")
            self.dp_shard = self.world_size // denom
        if self.dp_shard < 1:
            raise ValueError("dp_shard must be -1 or >= 1")
        prod = self.dp_replicate * self.dp_shard * self.cp * self.tp * self.pp
        if prod != self.world_size:
            raise ValueError(
                f"dp_replicate({self.dp_replicate})*dp_shard({self.dp_shard})*cp({self.cp})*tp({self.tp})*"
                f"pp({self.pp}) = {prod} != world_size({self.world_size})"
            )
        if self.ep > 1:
            if self.etp not in (1, self.tp):
                raise ValueError("etp must be 1 or equal to tp")
            span = self.dp_shard * self.cp * self.tp
            if span % (self.ep * self.etp):
                raise ValueError(f"ep*etp ({self.ep * self.etp}) must divide dp_shard*cp*tp ({span})")

    # ---- degrees --------------------------------------------------------
    @property
    def efsdp(self) -> int:
        return self.dp_shard * self.cp * self.tp // (self.ep * self.etp)

    @property
    def dp_enabled(self) -> bool:
        return self.dp_replicate > 1 or self.dp_shard > 1

    @property
    def dp_replicate_enabled(self) -> bool:
        return self.dp_replicate > 1

    @property
    def dp_shard_enabled(self) -> bool:
        return self.dp_shard > 1

    @property
    def fsdp_enabled(self) -> bool:
        return self.dp_shard > 1 or self.cp > 1

    @property
    def cp_enabled(self) -> bool:
        return self.cp > 1

    @property
    def dp_cp_enabled(self) -> bool:
        return self.dp_enabled or self.cp_enabled

    @property
    def tp_enabled(self) -> bool:
        return self.tp > 1

    @property
    def pp_enabled(self) -> bool:
        return self.pp > 1

    @property
    def ep_enabled(self) -> bool:
        return self.ep > 1

    @property
    def etp_enabled(self) -> bool:
        return self.etp > 1

    @property
    def seq_len_divisor(self) -> int:
        return self.tp * 2 * self.cp

    @property
    def non_data_parallel_size(self) -> int:
        return self.cp * self.tp * self.pp

    # ---- meshes ---------------------------------------------------------
    _DENSE = ("pp", "dp_replicate", "dp_shard", "cp", "tp")
    _SPARSE = ("pp", "dp_replicate", "efsdp", "ep", "etp")
    _FLAT = {
        "fsdp": ("dp_shard", "cp"),
        "batch": ("dp_replicate", "dp_shard"),
        "loss": ("dp_replicate", "dp_shard", "cp"),
        "dp_cp": ("dp_replicate", "dp_shard", "cp"),
        "dp": ("dp_replicate", "dp_shard"),
    }

    def mesh_size(self, name: str) -> int:
        if name in self._FLAT:
            n = 1
            for d in self._FLAT[name]:
                n *= self.mesh_size(d)
            return n
        return int(getattr(self, name))

    def _device_type(self) -> str:
        import torch.distributed as dist

        if dist.is_initialized() and dist.get_backend() == "gloo":
            return "cpu"
        return "cuda" if torch.cuda.is_available() else "cpu"

    def _root(self, kind: str):
        if kind not in self._meshes:
            from torch.distributed.device_mesh import DeviceMesh

            names = self._DENSE if kind == "dense" else self._SPARSE
            shape = tuple(self.mesh_size(n) for n in names)
            ranks = torch.arange(self.world_size).view(shape)
            self._meshes[kind] = DeviceMesh(self._device_type(), ranks, mesh_dim_names=names)
        return self._meshes[kind]

    def get_mesh(self, names: str | list[str]):
        key = names if isinstance(names, str) else "+".join(names)
        if key in self._meshes:
            return self._meshes[key]
        if isinstance(names, str) and names in self._FLAT:
            sub = self._root("dense")[self._FLAT[names]]
            m = sub._flatten(names) if len(self._FLAT[names]) > 1 else sub
        elif isinstance(names, str):
            root = self._root("sparse" if names in ("efsdp", "ep", "etp") else "dense")
            m = root[names]
        else:
            sparse = any(n in ("efsdp", "ep", "etp") for n in names)
            for n in names:
                if n in self._FLAT:
                    self.get_mesh(n)  # registers the flattened dim on the root mesh
            m = self._root("sparse" if sparse else "dense")[tuple(names)]
        self._meshes[key] = m
        return m

    def get_optional_mesh(self, names: str | list[str]):
        size = 1
        for n in ([names] if isinstance(names, str) else names):
            size *= self.mesh_size(n)
        return None if size == 1 else self.get_mesh(names)

    def build_mesh(self):
        return self._root("dense")

    @property
    def world_mesh(self):
        return self._root("dense")
