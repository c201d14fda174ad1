"""Non-finite canaries: name the first module whose forward output holds a NaN or Inf.

Debugging aid (``--debug.nonfinite-check``): a forward hook on every module checks its
tensor outputs and raises ``FloatingPointError`` with the module's name, so a divergence
is traced to the layer that produced it instead of surfacing as a NaN loss.  Each check is
a device-to-host read; leave it off for performance runs."""
from __future__ import annotations

import torch
import torch.nn as nn


def _tensors(out):
    if torch.is_tensor(out):
        yield out
    elif isinstance(out, (list, tuple)):
        for o in out:
            yield from _tensors(o)
    elif isinstance(out, dict):
        for o in out.values():
            yield from _tensors(o)


def install_nonfinite_hooks(model: nn.Module) -> list:
    """Register the hooks; returns their handles (``h.remove()`` to take them off)."""
    handles = []
    for name, mod in model.named_modules():
        def hook(m, inp, out, name=name or type(model).__name__):
            for t in _tensors(out):
                if t.is_floating_point() and t.device.type != "meta" and not bool(torch.isfinite(t).all()):
                    raise FloatingPointError(f"non-finite values in the output of {name} ({type(m).__name__})")
        handles.append(mod.register_forward_hook(hook))
    return handles
