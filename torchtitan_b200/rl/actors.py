"""A minimal actor runtime for the RL loop: one process per actor, method calls over a pipe.

Role parity: the reference runs its generator, trainer and grader as Monarch actors
(``experiments/rl/simple_grpo_sum_digits.py``, ``actors/*.py``), each on its own GPU mesh.
Monarch is not available here, so an actor is a ``torch.multiprocessing`` (spawn) child that
builds an object from ``(cls, args, kwargs)`` and serves ``(method, args, kwargs)`` requests
in order.  Tensors in arguments and results travel through torch's shared-memory reductions
(CPU shared memory, CUDA IPC handles), so weight pushes do not pickle tensor data.

``ActorHandle.<method>(...)`` returns an ``asyncio`` awaitable; ``call_sync`` blocks.  Calls
to one actor are serialised (one request in flight per actor); different actors run in
parallel.  A child that raises sends the traceback back, and the awaiting caller re-raises it
as :class:`ActorError`.  ``gpus`` pins the child to devices through ``CUDA_VISIBLE_DEVICES``
before it imports CUDA state (the reference's ``Provisioner``).
"""
from __future__ import annotations

import asyncio
import os
import threading
import traceback
from typing import Any

import torch.multiprocessing as mp


class ActorError(RuntimeError):
    pass


def _serve(conn, cls, args, kwargs, env):
    os.environ.update(env)
    try:
        obj = cls(*args, **kwargs)
        conn.send(("ok", None))
    except Exception:  # noqa: BLE001
        conn.send(("err", traceback.format_exc()))
        return
    while True:
        try:
            msg = conn.recv()
        except EOFError:
            return
        if msg is None:
            getattr(obj, "close", lambda: None)()
            conn.send(("ok", None))
            return
        name, a, k = msg
        try:
            conn.send(("ok", getattr(obj, name)(*a, **k)))
        except Exception:  # noqa: BLE001
            conn.send(("err", traceback.format_exc()))


class ActorHandle:
    def __init__(self, cls: type, *args: Any, gpus: list[int] | None = None, env: dict | None = None,
                 **kwargs: Any):
        ctx = mp.get_context("spawn")
        self._conn, child = ctx.Pipe()
        e = dict(env or {})
        if gpus is not None:
            e["CUDA_VISIBLE_DEVICES"] = ",".join(str(g) for g in gpus)
        self._proc = ctx.Process(target=_serve, args=(child, cls, args, kwargs, e), daemon=True)
        self._proc.start()
        self._lock = threading.Lock()
        self.name = cls.__name__
        status, tb = self._conn.recv()
        if status != "ok":
            self._proc.join(5)
            raise ActorError(f"actor {self.name} failed to start:\n{tb}")

    def call_sync(self, method: str, *args: Any, **kwargs: Any) -> Any:
        with self._lock:
            self._conn.send((method, args, kwargs))
            status, val = self._conn.recv()
        if status != "ok":
            raise ActorError(f"{self.name}.{method} raised:\n{val}")
        return val

    async def call(self, method: str, *args: Any, **kwargs: Any) -> Any:
        return await asyncio.to_thread(self.call_sync, method, *args, **kwargs)

    def __getattr__(self, method: str):
        if method.startswith("_"):
            raise AttributeError(method)
        return lambda *a, **k: self.call(method, *a, **k)

    def stop(self, timeout: float = 30.0) -> None:
        if self._proc.is_alive():
            try:
                with self._lock:
                    self._conn.send(None)
                    self._conn.recv()
            except (EOFError, BrokenPipeError, OSError):
                pass
            self._proc.join(timeout)
            if self._proc.is_alive():
                self._proc.terminate()
                self._proc.join(5)


class Provisioner:
    """Hands out disjoint GPU ranges to actors (the trainer and the generator on separate GPUs)."""

    def __init__(self, total_gpus: int):
        self.total = total_gpus
        self.next = 0

    def allocate(self, n: int) -> list[int]:
        if self.next + n > self.total:
            raise RuntimeError(f"asked for {n} GPUs, {self.total - self.next} of {self.total} left")
        ids = list(range(self.next, self.next + n))
        self.next += n
        return ids
