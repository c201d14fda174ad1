"""``--module M --config C [--section.key value ...]`` command-line front end.

``M`` names a package under ``torchtitan_b200.models`` (or a dotted import
path); its ``config_registry`` module exposes functions returning a fully
populated ``Trainer.Config``.  Everything else on the command line is parsed by
tyro as an override of that config (reference behaviour:
``torchtitan/config/manager.py:34-150``).
"""
from __future__ import annotations

import importlib
import sys
from typing import Any

import tyro

_SHORT_MODULES = ("llama3", "kimi_linear", "deepseek_v3", "qwen3", "llama4", "gpt_oss", "attention_residual", "hf_transformers")


def split_module_and_config(args: list[str]) -> tuple[str | None, str | None, list[str]]:
    """Pull ``--module`` / ``--config`` (both ``--x v`` and ``--x=v`` forms) out of argv."""
    module = config = None
    rest: list[str] = []
    it = iter(range(len(args)))
    i = 0
    while i < len(args):
        a = args[i]
        key = None
        for name in ("--module", "--config"):
            if a == name:
                if i + 1 >= len(args):
                    raise ValueError(f"{name} requires a value")
                key, val = name, args[i + 1]
                i += 1
            elif a.startswith(name + "="):
                key, val = name, a.split("=", 1)[1]
        if key == "--module":
            module = val
        elif key == "--config":
            config = val
        else:
            rest.append(a)
        i += 1
    del it
    return module, config, rest


def import_config_registry(module: str):
    candidates = []
    if module in ("graph", "graph_trainer"):  # the graph trainer's registry
        candidates.append("torchtitan_b200.graph.config_registry")
    if module in _SHORT_MODULES or "." not in module:
        candidates.append(f"torchtitan_b200.models.{module}.config_registry")
    candidates += [f"{module}.config_registry", module]
    errors = []
    for c in candidates:
        try:
            return importlib.import_module(c)
        except ImportError as e:  # try the next spelling
            errors.append(f"{c}: {e}")
    raise ImportError(f"cannot import a config registry for '{module}':\n  " + "\n  ".join(errors))


def load_registered_config(module: str, config: str):
    reg = import_config_registry(module)
    fn = getattr(reg, config, None)
    if fn is None or not callable(fn):
        avail = sorted(n for n in dir(reg) if not n.startswith("_") and callable(getattr(reg, n)) and n[0].islower())
        raise ValueError(f"config function '{config}' not in {reg.__name__}; available: {avail}")
    return fn()


class ConfigManager:
    """Parses a job config: registry defaults < command-line overrides."""

    def parse_args(self, args: list[str] | None = None) -> Any:
        args = list(sys.argv[1:] if args is None else args)
        module, config, rest = split_module_and_config(args)
        if module is None or config is None:
            raise ValueError("both --module and --config are required, e.g. --module llama3 --config llama3_debugmodel")
        loaded = load_registered_config(module, config)
        self.config = tyro.cli(type(loaded), args=rest, default=loaded)
        self._validate(self.config)
        return self.config

    @staticmethod
    def _validate(cfg: Any) -> None:
        tr = getattr(cfg, "training", None)
        if tr is not None and tr.seq_len <= 0:
            raise ValueError("training.seq_len must be positive")


if __name__ == "__main__":  # python -m torchtitan_b200.config.manager --module ... --config ...
    import json

    c = ConfigManager().parse_args()
    print(json.dumps(c.to_dict(), indent=2))
