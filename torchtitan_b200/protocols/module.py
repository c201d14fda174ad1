"""Module protocol (parity: ``torchtitan/protocols/module.py:23-172``).

A ``Module`` is an ``nn.Module`` that knows how to initialise its own state:

* ``param_init``: optional ``{param_name: fn(tensor) -> None}`` table applied
  to this module's *direct* parameters by ``init_states``;
* ``init_self(buffer_device)``: hook for anything else the module owns
  (buffers, tables);
* ``init_states(buffer_device)``: recursive -- children first, then this
  module's ``param_init`` entries and ``init_self``.  Children that are plain
  ``nn.Module``s are initialised with their ``reset_parameters`` if they have one.

``Module.from_nn_module(mod, param_init)`` turns an existing module instance
into a protocol module in place (its class is swapped for a subclass that
also derives from ``Module``), so third-party layers join the recursive
initialisation without being rewritten.
"""
from __future__ import annotations

from collections.abc import Callable

import torch
import torch.nn as nn

_SUBCLASSES: dict[type, type] = {}


class Module(nn.Module):
    param_init: dict[str, Callable[[torch.Tensor], None]] | None = None

    def init_self(self, buffer_device: torch.device | None = None) -> None:
        """Initialise what ``param_init`` does not cover (override as needed)."""

    @torch.no_grad()
    def init_states(self, buffer_device: torch.device | None = None) -> None:
        for child in self.children():
            if isinstance(child, Module):
                child.init_states(buffer_device)
            else:
                _init_plain(child, buffer_device)
        for name, fn in (self.param_init or {}).items():
            p = self._parameters.get(name)
            if p is None:
                raise KeyError(f"{type(self).__name__}.param_init names '{name}', which is not a direct parameter")
            fn(p)
        self.init_self(buffer_device)

    @staticmethod
    def from_nn_module(mod: nn.Module, param_init: dict[str, Callable[[torch.Tensor], None]] | None = None
                       ) -> "Module":
        cls = type(mod)
        if not isinstance(mod, Module):
            sub = _SUBCLASSES.get(cls)
            if sub is None:
                sub = type(cls.__name__, (cls, Module), {})
                _SUBCLASSES[cls] = sub
            mod.__class__ = sub
        if param_init is not None:
            mod.param_init = dict(param_init)
        return mod  # type: ignore[return-value]


def _init_plain(mod: nn.Module, buffer_device) -> None:
    if hasattr(mod, "reset_parameters"):
        mod.reset_parameters()
    for child in mod.children():
        if isinstance(child, Module):
            child.init_states(buffer_device)
        else:
            _init_plain(child, buffer_device)
