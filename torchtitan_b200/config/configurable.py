"""Configurable components.

Every swappable part of the trainer is a ``Configurable`` with a nested
``Config`` dataclass.  ``Config.build(**runtime)`` constructs the owning class,
passing runtime-only objects (meshes, model parts, tokenizers) as keyword
arguments that must not collide with config fields.

Interface parity: ``torchtitan/config/configurable.py:15-113`` in the
reference (nested kw_only/slots Config, auto-wired ``build``).  The
implementation here is independent: ownership is recorded by
``__init_subclass__`` and validation happens once per class.
"""
from __future__ import annotations

import dataclasses
from dataclasses import dataclass
from typing import Any, ClassVar


def _to_plain(value: Any) -> Any:
    if hasattr(value, "to_dict") and callable(value.to_dict):
        return value.to_dict()
    if dataclasses.is_dataclass(value) and not isinstance(value, type):
        return {f.name: _to_plain(getattr(value, f.name)) for f in dataclasses.fields(value)}
    if isinstance(value, (list, tuple)):
        return [_to_plain(v) for v in value]
    if isinstance(value, dict):
        return {str(k): _to_plain(v) for k, v in value.items()}
    if value is None or isinstance(value, (bool, int, float, str)):
        return value
    return repr(value)


class Configurable:
    """Base for every component that is built from a ``Config``."""

    @dataclass(kw_only=True, slots=True)
    class Config:
        _owner: ClassVar[type | None] = None

        def to_dict(self) -> dict:
            return {f.name: _to_plain(getattr(self, f.name)) for f in dataclasses.fields(self)}

        def build(self, **runtime: Any):
            owner = type(self)._owner
            if owner is None:
                raise NotImplementedError(f"{type(self).__qualname__} is not owned by a Configurable")
            names = {f.name for f in dataclasses.fields(self)}
            clash = names.intersection(runtime)
            if clash:
                raise ValueError(f"build() runtime kwargs {sorted(clash)} shadow config fields")
            return owner(config=dataclasses.replace(self), **runtime)

    def __init_subclass__(cls, **kw):
        super().__init_subclass__(**kw)
        cfg = cls.__dict__.get("Config")
        if cfg is None or not isinstance(cfg, type) or not issubclass(cfg, Configurable.Config):
            return
        if "__slots__" not in cfg.__dict__:
            raise TypeError(f"{cls.__name__}.Config must be @dataclass(kw_only=True, slots=True)")
        for f in dataclasses.fields(cfg):
            if f.init and not f.kw_only:
                raise TypeError(f"{cls.__name__}.Config.{f.name} must be keyword-only")
        cfg._owner = cls
