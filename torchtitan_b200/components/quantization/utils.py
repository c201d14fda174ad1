"""Which linears a quantization converter may swap (parity: reference
``quantization/utils.py:10-27``): dims divisible by the format's block, FQN not
in the exclusion list (the output head by default)."""
from __future__ import annotations

import torch.nn as nn


def module_filter(fqn: str, mod: nn.Module, *, divisor: int = 16, filter_fqns: list[str] = ()) -> bool:
    from torchtitan_b200.models.common import Linear

    if not isinstance(mod, Linear):
        return False
    if any(f in fqn for f in filter_fqns):
        return False
    return mod.in_features % divisor == 0 and mod.out_features % divisor == 0


def swap_linears(model: nn.Module, new_cls: type, divisor: int, filter_fqns: list[str], **attrs) -> int:
    n = 0
    for fqn, mod in model.named_modules():
        if module_filter(fqn, mod, divisor=divisor, filter_fqns=filter_fqns):
            mod.__class__ = new_cls
            for k, v in attrs.items():
                setattr(mod, k, v)
            n += 1
    return n
