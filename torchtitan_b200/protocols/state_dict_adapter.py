"""Native <-> Hugging Face state-dict mapping.

Parity: ``torchtitan/protocols/state_dict_adapter.py:20-120``.  An adapter maps
this framework's FQNs (which equal the reference's) to HF names and back, and
can read ``model.safetensors.index.json`` to know which HF file holds a key.
"""
from __future__ import annotations

import json
import os
import re
from abc import ABC, abstractmethod
from typing import Any


class BaseStateDictAdapter(ABC):
    fqn_to_index_mapping: dict[str, int] | None = None

    @abstractmethod
    def to_hf(self, state_dict: dict[str, Any]) -> dict[str, Any]:
        ...

    @abstractmethod
    def from_hf(self, hf_state_dict: dict[str, Any]) -> dict[str, Any]:
        ...


class StateDictAdapter(BaseStateDictAdapter):
    """Regex-table adapter: ``from_hf_map`` maps HF patterns (with ``{}`` for
    the layer index) to native patterns."""

    from_hf_map: dict[str, str | None] = {}

    def __init__(self, model_args: Any = None, hf_assets_path: str | None = None):
        self.model_args = model_args
        self.fqn_to_index_mapping = None
        if hf_assets_path:
            idx = os.path.join(hf_assets_path, "model.safetensors.index.json")
            if os.path.exists(idx):
                with open(idx) as f:
                    wm = json.load(f)["weight_map"]
                self.fqn_to_index_mapping = {
                    k: int(re.search(r"(\d+)-of", v).group(1)) if re.search(r"(\d+)-of", v) else 1
                    for k, v in wm.items()
                }
        self._to_hf = {v: k for k, v in self.from_hf_map.items() if v is not None}

    @staticmethod
    def _apply(name: str, table: dict[str, str | None]) -> str | None:
        if name in table:
            return table[name]
        m = re.search(r"\.(\d+)\.", name)
        if m is None:
            return None
        key = name.replace(f".{m.group(1)}.", ".{}.", 1)
        tgt = table.get(key)
        return None if tgt is None else tgt.format(m.group(1))

    def to_hf(self, state_dict: dict[str, Any]) -> dict[str, Any]:
        out = {}
        for k, v in state_dict.items():
            nk = self._apply(k, self._to_hf)
            if nk is not None:
                out[nk] = self.to_hf_tensor(k, v)
        return out

    def from_hf(self, hf_state_dict: dict[str, Any]) -> dict[str, Any]:
        out = {}
        for k, v in hf_state_dict.items():
            nk = self._apply(k, self.from_hf_map)
            if nk is not None:
                out[nk] = self.from_hf_tensor(nk, v)
        return out

    def to_hf_tensor(self, native_key: str, t: Any) -> Any:
        return t

    def from_hf_tensor(self, native_key: str, t: Any) -> Any:
        return t
