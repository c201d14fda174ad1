"""Host-side watch on the device error word of the peer-memory collectives.

Every cross-GPU wait in ``dp_comm.cu`` (reduce-scatter, barriers -- also used
by the fused expert-parallel path) gives up after a bounded time and records
``[code, slot, epoch, source rank, value seen]``.  Besides the device copy it
writes them into a pinned host buffer registered here, so this module can see
a failure *while the GPU is still working through the queue*, with no CUDA
call: a daemon thread polls the buffer, logs the failure once, and sets a flag
the trainer checks between steps (it then raises instead of training on with
partial gradients).
"""
from __future__ import annotations

import threading
import time
from collections.abc import Callable

import torch

from torchtitan_b200.utils.logging import logger

_SINK: torch.Tensor | None = None
_WATCH: "ErrorWatchdog | None" = None

CODES = {71: "reduce-scatter wait", 72: "epoch barrier wait"}


def describe(word: list[int]) -> str:
    code, slot, epoch, src, seen = word[:5]
    return (f"{CODES.get(code, f'code {code}')} timed out: slot {slot}, waiting for epoch {epoch} from "
            f"rank {src}, flag seen {seen}")


class ErrorWatchdog:
    def __init__(self, sink: torch.Tensor, interval_s: float = 0.5,
                 on_error: Callable[[list[int]], None] | None = None):
        self.sink = sink
        self.interval_s = interval_s
        self.on_error = on_error
        self.error: list[int] | None = None
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._run, name="ttb-peer-watchdog", daemon=True)
        self._thread.start()

    def poll(self) -> list[int] | None:
        if self.error is None and int(self.sink[0]) != 0:
            self.error = [int(x) for x in self.sink.tolist()]
            logger.error(f"peer-memory collective: {describe(self.error)}")
            if self.on_error is not None:
                self.on_error(self.error)
        return self.error

    def reset(self) -> None:
        """Clear a reported failure (after it was handled) and resume watching."""
        self.sink.zero_()
        self.error = None
        if not self._thread.is_alive():
            self._stop.clear()
            self._thread = threading.Thread(target=self._run, name="ttb-peer-watchdog", daemon=True)
            self._thread.start()

    def _run(self) -> None:
        while not self._stop.wait(self.interval_s):
            if self.poll() is not None:
                return

    def stop(self) -> None:
        self._stop.set()


def install(ext=None, interval_s: float = 0.5) -> ErrorWatchdog:
    """Register the pinned error buffer with the kernels (once per process) and start the watch."""
    global _SINK, _WATCH
    if _WATCH is None:
        if ext is None:
            from torchtitan_b200.ops._ext import ext as _e

            ext = _e()
        _SINK = torch.zeros(8, dtype=torch.int32).pin_memory()
        ext.dp_set_error_sink(_SINK)
        _WATCH = ErrorWatchdog(_SINK, interval_s)
    return _WATCH


def current() -> ErrorWatchdog | None:
    return _WATCH
