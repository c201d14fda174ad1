"""Bitwise fingerprints of models, gradients and optimizer states (parity: reference
``tests/utils.py:14-122``), for determinism checks: two runs that should be identical
must give identical hashes, and a single flipped bit changes them.

Tensors are hashed in name order from their full (unsharded) values, so the digest
does not depend on how a model is sharded; bfloat16 and other dtypes are hashed from
their raw bytes."""
from __future__ import annotations

import hashlib
from collections.abc import Iterable

import torch


def _full(t: torch.Tensor) -> torch.Tensor:
    if type(t).__name__ == "DTensor":
        t = t.full_tensor()
    return t.detach().contiguous().cpu()


def tensor_bytes(t: torch.Tensor) -> bytes:
    t = _full(t)
    return t.reshape(-1).view(torch.uint8).numpy().tobytes() if t.numel() else b""


def hash_tensors(named: Iterable[tuple[str, torch.Tensor | None]]) -> str:
    h = hashlib.sha256()
    for name, t in sorted(named, key=lambda kv: kv[0]):
        h.update(name.encode())
        if t is None:
            h.update(b"<none>")
            continue
        h.update(str(t.dtype).encode() + str(tuple(t.shape)).encode())
        h.update(tensor_bytes(t))
    return h.hexdigest()


def hash_model(model: torch.nn.Module) -> str:
    return hash_tensors(model.named_parameters())


def hash_grads(model: torch.nn.Module) -> str:
    return hash_tensors((n, p.grad) for n, p in model.named_parameters())


def hash_optimizer(opt: torch.optim.Optimizer) -> str:
    items = []
    for i, (p, st) in enumerate(opt.state.items()):
        for k, v in st.items():
            if torch.is_tensor(v):
                items.append((f"{i}.{k}", v))
    return hash_tensors(items)
