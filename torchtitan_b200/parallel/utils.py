"""Process-group bring-up, determinism, scalar collectives and grad clipping.

Parity: ``torchtitan/distributed/utils.py`` -- ``init_distributed`` (NCCL with
flight recorder + async error handling env, or fake/local modes), PG timeout
tightening after step 1 (``:414-442``), ``set_determinism`` (seed broadcast,
deterministic algorithms), ``dist_sum/max/mean`` and ``clip_grad_norm_`` over
DTensor shards (``:446-591``).
"""
from __future__ import annotations

import contextlib
import datetime
import os
from typing import Any

import torch
import torch.distributed as dist

from torchtitan_b200.utils.logging import logger

try:
    from torch.distributed.tensor import DTensor, Replicate, Shard, Partial
except ImportError:  # pragma: no cover
    DTensor = ()  # type: ignore


def _ensure_env_single_process() -> None:
    os.environ.setdefault("RANK", "0")
    os.environ.setdefault("LOCAL_RANK", "0")
    os.environ.setdefault("WORLD_SIZE", "1")
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    if "MASTER_PORT" not in os.environ:
        import socket

        s = socket.socket()
        s.bind(("127.0.0.1", 0))
        os.environ["MASTER_PORT"] = str(s.getsockname()[1])
        s.close()


_LOCAL_TENSOR_MODE = None


def init_distributed(comm: Any, *, enable_cpu_backend: bool = False, base_folder: str = "",
                     backend: str | None = None) -> int:
    """Initialise the default process group and return the world size."""
    if dist.is_initialized():
        return dist.get_world_size()
    _ensure_env_single_process()
    mode = getattr(comm, "mode", "default")
    if mode == "fake_backend":
        from torch.testing._internal.distributed.fake_pg import FakeStore

        ws = int(os.environ.get("NGPU", os.environ["WORLD_SIZE"]))
        dist.init_process_group("fake", store=FakeStore(), rank=0, world_size=ws)
        return ws
    if mode == "local_tensor":
        # One process simulates every rank: a fake process group carries the collectives and
        # LocalTensorMode runs each rank's shard of every DTensor op numerically
        # (reference: distributed/utils.py:296-336). CPU debugging only; CUDA kernels of this
        # package have no LocalTensor dispatch, so the model falls back to PyTorch ops.
        from torch.distributed import _local_tensor
        from torch.testing._internal.distributed.fake_pg import FakeStore

        ws = int(os.environ.get("NGPU", os.environ["WORLD_SIZE"]))
        dist.init_process_group("fake", store=FakeStore(), rank=0, world_size=ws)
        lm = _local_tensor.LocalTensorMode(ws)
        lm.__enter__()
        global _LOCAL_TENSOR_MODE
        _LOCAL_TENSOR_MODE = lm
        return ws
    if backend is None:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
        if enable_cpu_backend and backend == "nccl":
            backend = "cuda:nccl,cpu:gloo"
    if "nccl" in backend:
        os.environ.setdefault("TORCH_NCCL_ASYNC_ERROR_HANDLING", "3")
        os.environ.setdefault("TORCH_FR_BUFFER_SIZE", str(getattr(comm, "trace_buf_size", 20000)))
        if getattr(comm, "trace_buf_size", 0) > 0:
            d = os.path.join(base_folder, getattr(comm, "save_traces_folder", "comm_traces"))
            os.environ.setdefault("TORCH_FR_DUMP_TEMP_FILE", os.path.join(d, getattr(comm, "save_traces_file_prefix", "rank_")))
    kw = {}
    if torch.cuda.is_available() and "nccl" in backend:
        kw["device_id"] = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    dist.init_process_group(backend, timeout=datetime.timedelta(seconds=getattr(comm, "init_timeout_seconds", 300)), **kw)
    return dist.get_world_size()


def set_pg_timeouts(timeout: datetime.timedelta, parallel_dims: Any = None) -> None:
    """Barrier, then shorten the default PG timeout (faster failure signal after warm-up)."""
    if not dist.is_initialized():
        return
    dist.barrier()
    if torch.cuda.is_available():
        torch.cuda.synchronize()
    try:
        from torch.distributed.distributed_c10d import _get_default_group, _set_pg_timeout

        _set_pg_timeout(timeout, _get_default_group())
        for m in (parallel_dims._meshes.values() if parallel_dims is not None else []):
            for g in (m.get_all_groups() if hasattr(m, "get_all_groups") else []):
                _set_pg_timeout(timeout, g)
    except Exception as e:  # older torch / fake PG
        logger.warning(f"could not tighten PG timeouts: {e}")


def _reduce(x: torch.Tensor | float, op, mesh: Any = None) -> float:
    t = x.detach().clone() if torch.is_tensor(x) else torch.tensor(float(x))
    if mesh is not None and dist.is_initialized():
        if t.device.type == "cpu" and dist.get_backend(mesh.get_group()) not in ("gloo", "fake") \
                and torch.cuda.is_available():
            t = t.cuda()
        dist.all_reduce(t, op=op, group=mesh.get_group())
    return t


def dist_sum(x, mesh: Any = None):
    return _reduce(x, dist.ReduceOp.SUM, mesh)


def dist_max(x, mesh: Any = None):
    return _reduce(x, dist.ReduceOp.MAX, mesh)


def dist_mean(x, mesh: Any = None):
    t = _reduce(x, dist.ReduceOp.SUM, mesh)
    return t / (mesh.size() if mesh is not None else 1)


BATCH_INVARIANT_NCCL_ENV = {"NCCL_ALGO": "Ring", "NCCL_PROTO": "Simple", "NCCL_MIN_NCHANNELS": "1",
                            "NCCL_MAX_NCHANNELS": "1", "NCCL_NVLS_ENABLE": "0", "NCCL_COLLNET_ENABLE": "0"}


def apply_batch_invariant_env() -> dict[str, str]:
    """Fix NCCL's reduction order (ring, one channel, simple protocol, no in-switch or
    in-network reduction) so collectives give bit-identical results whatever the
    message size (parity: reference ``distributed/utils.py:218-273``).  Must run before
    the process group exists.  This framework's GEMM, attention and cross-entropy
    kernels reduce each output element in a fixed order with no split-K, so they are
    batch-invariant already."""
    for k, v in BATCH_INVARIANT_NCCL_ENV.items():
        os.environ[k] = v
    return dict(BATCH_INVARIANT_NCCL_ENV)


def set_determinism(parallel_dims: Any, device: torch.device, debug: Any,
                    distinct_seed_mesh_dims: list[str] | None = None) -> None:
    if debug.deterministic:
        torch.use_deterministic_algorithms(True, warn_only=debug.deterministic_warn_only)
        torch.backends.cudnn.deterministic = True
        torch.backends.cudnn.benchmark = False
        os.environ["CUBLAS_WORKSPACE_CONFIG"] = ":4096:8"
    if debug.detect_anomaly:
        torch.autograd.set_detect_anomaly(True)
    seed = debug.seed
    if seed is None and dist.is_initialized() and dist.get_world_size() > 1:
        t = torch.randint(0, 2**31 - 1, (1,), dtype=torch.int64)
        if dist.get_backend() == "nccl":
            t = t.to(device)
        dist.broadcast(t, src=0)
        seed = int(t.item())
    if seed is None:
        return
    # distinct seeds along e.g. pp so stages draw different init streams
    offset = 0
    if distinct_seed_mesh_dims and parallel_dims is not None:
        stride = 1
        for d in distinct_seed_mesh_dims:
            m = parallel_dims.get_optional_mesh(d)
            if m is not None:
                offset += m.get_local_rank() * stride
                stride *= m.size()
    torch.manual_seed(seed + offset)
    if torch.cuda.is_available():
        torch.cuda.manual_seed_all(seed + offset)


@torch.no_grad()
def clip_grad_norm_(parameters, max_norm: float, norm_type: float = 2.0, foreach: bool = True,
                    pp_mesh: Any = None, ep_enabled: bool = False, defer_scaling: bool = False):
    """Global grad-norm (over DTensor shards, PP stages) and in-place clipping.

    Local squared norms are summed per (mesh, shard-dims) signature, reduced
    across the sharded mesh dims only (replicated dims hold equal copies),
    then summed, reduced across PP stages, and used to scale every grad.
    """
    grads = [p.grad for p in parameters if p.grad is not None]
    if not grads:
        return (torch.zeros(()), torch.zeros(())) if defer_scaling else torch.zeros(())
    assert norm_type == 2.0, "only the 2-norm is supported"
    per_sig: dict[Any, list[torch.Tensor]] = {}
    for g in grads:
        if isinstance(g, DTensor):
            shard_dims = tuple(i for i, p in enumerate(g.placements) if isinstance(p, (Shard, Partial)) or type(p).__name__.startswith("_Strided"))
            key = (id(g.device_mesh), shard_dims)
            per_sig.setdefault(key, [g.device_mesh, shard_dims, []])[2].append(g.to_local())
        else:
            per_sig.setdefault(("plain",), [None, (), []])[2].append(g)
    total = None
    for mesh, shard_dims, locs in per_sig.values():
        if locs[0].is_cuda:
            from torchtitan_b200.ops._ext import ext

            sq = ext().multi_sumsq([t if t.is_contiguous() else t.contiguous() for t in locs])
        else:
            norms = torch._foreach_norm([t.float() for t in locs], 2.0)
            sq = torch.stack(list(norms)).pow(2).sum()
        if mesh is not None:
            for d in shard_dims:
                dist.all_reduce(sq, group=mesh.get_group(d))
        total = sq if total is None else total + sq.to(total.device)
    if pp_mesh is not None:
        dist.all_reduce(total, group=pp_mesh.get_group())
    norm = total.sqrt()
    if defer_scaling:
        return norm, total  # the fused optimizer applies the clip coefficient itself
    if max_norm and max_norm > 0:
        locs = [g.to_local() if isinstance(g, DTensor) else g for g in grads]
        if locs[0].is_cuda and all(t.is_contiguous() for t in locs):
            from torchtitan_b200.ops._ext import ext

            ext().multi_clip_scale(locs, total.float().contiguous(), float(max_norm))
        else:
            coef = (max_norm / (norm + 1e-6)).clamp(max=1.0)
            torch._foreach_mul_(locs, coef.to(locs[0].device))
    return norm


def get_train_context(loss_parallel_enabled: bool = False):
    @contextlib.contextmanager
    def ctx():
        if loss_parallel_enabled:
            from torch.distributed.tensor.parallel import loss_parallel

            with loss_parallel():
                yield
        else:
            yield

    return ctx
