"""Device helpers: peak FLOPs table, garbage-collection control, dtype defaults.

Peak table follows the vendor dense (non-sparse) figures; B200 bf16 dense is
2.25e15 as in the reference (``torchtitan/tools/utils.py:126-129``).
"""
from __future__ import annotations

import contextlib
import gc
import time

import torch

from .logging import logger

device_type = "cuda" if torch.cuda.is_available() else "cpu"
device_module = torch.cuda if device_type == "cuda" else None

_PEAK_BF16 = [
    ("B200", 2.25e15),
    ("GB200", 2.5e15),
    ("H200", 989e12),
    ("H100 PCIe", 756e12),
    ("H100", 989e12),
    ("A100", 312e12),
    ("L40S", 362e12),
]


def get_peak_flops(device_name: str, dtype: str = "bf16") -> float:
    mult = {"bf16": 1.0, "fp8": 2.0, "mxfp8": 2.0, "fp4": 4.0}[dtype]
    for key, val in _PEAK_BF16:
        if key in device_name:
            return val * mult
    logger.warning(f"peak FLOPs unknown for '{device_name}', assuming B200")
    return 2.25e15 * mult


class GarbageCollection:
    """Disable automatic GC and collect every ``gc_freq`` steps (avoids stragglers)."""

    def __init__(self, gc_freq: int = 1000, debug: bool = False):
        assert gc_freq > 0
        self.gc_freq = gc_freq
        self.debug = debug
        gc.disable()
        self.collect("initial gc")

    def run(self, step: int) -> None:
        if self.debug:
            gc.collect(1)
        elif step > 1 and step % self.gc_freq == 0:
            self.collect("periodic gc")

    @staticmethod
    def collect(reason: str, generation: int = 1) -> None:
        t0 = time.monotonic()
        gc.collect(generation)
        logger.debug(f"[GC] {reason} {time.monotonic() - t0:.2f}s")


@contextlib.contextmanager
def set_default_dtype(dtype: torch.dtype):
    old = torch.get_default_dtype()
    torch.set_default_dtype(dtype)
    try:
        yield
    finally:
        torch.set_default_dtype(old)


class Color:
    black = "\033[30m"; red = "\033[31m"; green = "\033[32m"; yellow = "\033[33m"
    blue = "\033[34m"; magenta = "\033[35m"; cyan = "\033[36m"; white = "\033[37m"; reset = "\033[39m"


class NoColor:
    black = red = green = yellow = blue = magenta = cyan = white = reset = ""
