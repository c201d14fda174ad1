"""FLUX.1 text-to-image rectified-flow transformer: flavors and the ``ModelSpec``
registry (parity: reference ``models/flux/__init__.py``; FLUX.1 dev/schnell sizes)."""
from __future__ import annotations

import copy

from torchtitan_b200.components.loss import build_mse_loss
from torchtitan_b200.protocols import ModelSpec

from .model import FluxModel, FluxModelArgs
from .parallelize import parallelize_flux

A = FluxModelArgs
flux_args = {
    "flux-debug": A(hidden_size=1536, num_heads=12, depth=2, depth_single_blocks=2),
    "flux-schnell": A(),
    "flux-dev": A(),
}


def model_registry(flavor: str) -> ModelSpec:
    if flavor not in flux_args:
        raise ValueError(f"unknown flux flavor '{flavor}', available: {sorted(flux_args)}")
    from .state_dict_adapter import FluxStateDictAdapter

    return ModelSpec(name="flux", flavor=flavor, model=copy.deepcopy(flux_args[flavor]),
                     parallelize_fn=parallelize_flux, pipelining_fn=None, build_loss_fn=build_mse_loss,
                     state_dict_adapter=FluxStateDictAdapter)


__all__ = ["FluxModel", "FluxModelArgs", "flux_args", "model_registry"]
