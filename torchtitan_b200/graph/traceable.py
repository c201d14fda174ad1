"""The sm_100a kernels as registered operators, so ``make_fx`` records them as graph nodes.

Eager code calls the extension through ``ops._ext.ext().<kernel>(...)`` from inside
``autograd.Function`` s.  A pybind call is opaque to tracing (under fake tensors it would
even try to read a data pointer), so while a step is traced :func:`traceable_kernels` makes
``ext()`` return :data:`_NS`, whose attributes are ``torch.library`` custom ops with shape
functions.  Running the traced graph then calls the same kernels through those ops.

Covered: every kernel of the dense decoder step (GEMM, attention forward/backward, RMSNorm,
RoPE, SwiGLU, cross entropy) and of the routed experts (routing selection, row gathers, grouped
GEMMs, dispatch / combine).  Any other attribute falls through to the extension itself,
which fails loudly under fake tensors.
"""
from __future__ import annotations

import contextlib
import importlib
from typing import Iterator

import torch

from torchtitan_b200.ops import _ext


def _C():
    return importlib.import_module("torchtitan_b200._C")


@torch.library.custom_op("tt_b200_graph::rmsnorm_fwd", mutates_args=())
def rmsnorm_fwd(x: torch.Tensor, w: torch.Tensor, eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    y, rstd = _C().rmsnorm_fwd(x, w, eps)
    return y, rstd


@rmsnorm_fwd.register_fake
def _(x, w, eps):
    return torch.empty_like(x), x.new_empty((x.shape[0],), dtype=torch.float32)


@torch.library.custom_op("tt_b200_graph::rmsnorm_bwd", mutates_args=())
def rmsnorm_bwd(dy: torch.Tensor, x: torch.Tensor, w: torch.Tensor,
                rstd: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    dx, dw = _C().rmsnorm_bwd(dy, x, w, rstd)
    return dx, dw


@rmsnorm_bwd.register_fake
def _(dy, x, w, rstd):
    return torch.empty_like(x), x.new_empty((x.shape[1],), dtype=torch.float32)


@torch.library.custom_op("tt_b200_graph::rope", mutates_args=())
def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, inverse: bool) -> torch.Tensor:
    return _C().rope(x, cos, sin, inverse)


@rope.register_fake
def _(x, cos, sin, inverse):
    return torch.empty_like(x)


@torch.library.custom_op("tt_b200_graph::swiglu_fwd", mutates_args=())
def swiglu_fwd(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    return _C().swiglu_fwd(a, b)


@swiglu_fwd.register_fake
def _(a, b):
    return torch.empty_like(a)


@torch.library.custom_op("tt_b200_graph::swiglu_bwd", mutates_args=())
def swiglu_bwd(dy: torch.Tensor, a: torch.Tensor, b: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    da, db = _C().swiglu_bwd(dy, a, b)
    return da, db


@swiglu_bwd.register_fake
def _(dy, a, b):
    return torch.empty_like(a), torch.empty_like(b)


@torch.library.custom_op("tt_b200_graph::ce_fwd", mutates_args=())
def ce_fwd(logits: torch.Tensor, labels: torch.Tensor, ignore_index: int) -> tuple[torch.Tensor, torch.Tensor]:
    loss, lse = _C().ce_fwd(logits, labels, ignore_index)
    return loss, lse


@ce_fwd.register_fake
def _(logits, labels, ignore_index):
    return logits.new_empty((), dtype=torch.float32), logits.new_empty((logits.shape[0],), dtype=torch.float32)


@torch.library.custom_op("tt_b200_graph::ce_bwd", mutates_args=())
def ce_bwd(logits: torch.Tensor, labels: torch.Tensor, lse: torch.Tensor, gscale: torch.Tensor,
           ignore_index: int) -> torch.Tensor:
    return _C().ce_bwd(logits, labels, lse, gscale, ignore_index)


@ce_bwd.register_fake
def _(logits, labels, lse, gscale, ignore_index):
    return torch.empty_like(logits)


@torch.library.custom_op("tt_b200_graph::attn_bwd", mutates_args=())
def attn_bwd(dout: torch.Tensor, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, o: torch.Tensor,
             lse: torch.Tensor, causal: bool, scale: float, dlse: torch.Tensor | None = None,
             doc_start: torch.Tensor | None = None,
             doc_end: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    dq, dk, dv = _C().attn_bwd(dout, q, k, v, o, lse, causal, scale, dlse=dlse, doc_start=doc_start,
                               doc_end=doc_end)
    return dq, dk, dv


@attn_bwd.register_fake
def _(dout, q, k, v, o, lse, causal, scale, dlse=None, doc_start=None, doc_end=None):
    return torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)


@torch.library.custom_op("tt_b200_graph::router_topk", mutates_args=())
def router_topk(logits: torch.Tensor, bias: torch.Tensor | None, top_k: int, sigmoid: bool, n_groups: int,
                limit_groups: int) -> tuple[torch.Tensor, torch.Tensor]:
    idx, counts = _C().router_topk(logits, bias, top_k, sigmoid, n_groups, limit_groups)
    return idx, counts


@router_topk.register_fake
def _(logits, bias, top_k, sigmoid, n_groups, limit_groups):
    return (logits.new_empty((logits.shape[0], top_k), dtype=torch.int64),
            logits.new_empty((logits.shape[1],), dtype=torch.int32))


@torch.library.custom_op("tt_b200_graph::gather_rows", mutates_args=())
def gather_rows(src: torch.Tensor, idx: torch.Tensor) -> torch.Tensor:
    return _C().gather_rows(src, idx)


@gather_rows.register_fake
def _(src, idx):
    return src.new_empty((idx.shape[0], src.shape[1]))


@torch.library.custom_op("tt_b200_graph::gemm_grouped_rows", mutates_args=())
def gemm_grouped_rows(a: torch.Tensor, b: torch.Tensor, tile_group: torch.Tensor, n_out: int, b_group_rows: int,
                      b_mn: bool) -> torch.Tensor:
    return _C().gemm_grouped_rows(a, b, tile_group, n_out, b_group_rows, b_mn)


@gemm_grouped_rows.register_fake
def _(a, b, tile_group, n_out, b_group_rows, b_mn):
    return a.new_empty((a.shape[0], n_out))


@torch.library.custom_op("tt_b200_graph::gemm_grouped_k", mutates_args=())
def gemm_grouped_k(a: torch.Tensor, b: torch.Tensor, kstart: torch.Tensor, klen: torch.Tensor) -> torch.Tensor:
    return _C().gemm_grouped_k(a, b, kstart, klen)


@gemm_grouped_k.register_fake
def _(a, b, kstart, klen):
    return a.new_empty((kstart.shape[0], a.shape[1], b.shape[1]))


@torch.library.custom_op("tt_b200_graph::moe_combine_fwd", mutates_args=())
def moe_combine_fwd(base: torch.Tensor | None, y: torch.Tensor, pos: torch.Tensor,
                    w: torch.Tensor | None) -> torch.Tensor:
    return _C().moe_combine_fwd(base, y, pos, w)


@moe_combine_fwd.register_fake
def _(base, y, pos, w):
    return y.new_empty((pos.shape[0], y.shape[1]))


@torch.library.custom_op("tt_b200_graph::moe_combine_bwd", mutates_args=())
def moe_combine_bwd(dout: torch.Tensor, y: torch.Tensor, pos: torch.Tensor, token_of: torch.Tensor,
                    scale: torch.Tensor | None, need_dw: bool) -> tuple[torch.Tensor, torch.Tensor]:
    dy, dw = _C().moe_combine_bwd(dout, y, pos, token_of, scale, need_dw)
    return dy, dw


@moe_combine_bwd.register_fake
def _(dout, y, pos, token_of, scale, need_dw):
    shape = tuple(pos.shape) if need_dw else (0, 0)
    return torch.empty_like(y), y.new_empty(shape, dtype=torch.float32)


class _TraceableKernels:
    """Stand-in for the extension module while tracing: the dense-step kernels as custom ops."""

    rmsnorm_fwd = staticmethod(lambda x, w, eps: torch.ops.tt_b200_graph.rmsnorm_fwd(x, w, float(eps)))
    rmsnorm_bwd = staticmethod(lambda dy, x, w, rstd: torch.ops.tt_b200_graph.rmsnorm_bwd(dy, x, w, rstd))
    rope = staticmethod(lambda x, cos, sin, inverse: torch.ops.tt_b200_graph.rope(x, cos, sin, bool(inverse)))
    swiglu_fwd = staticmethod(lambda a, b: torch.ops.tt_b200_graph.swiglu_fwd(a, b))
    swiglu_bwd = staticmethod(lambda dy, a, b: torch.ops.tt_b200_graph.swiglu_bwd(dy, a, b))
    ce_fwd = staticmethod(lambda lg, lb, ii: torch.ops.tt_b200_graph.ce_fwd(lg, lb, int(ii)))
    ce_bwd = staticmethod(lambda lg, lb, lse, g, ii: torch.ops.tt_b200_graph.ce_bwd(lg, lb, lse, g, int(ii)))
    gemm = staticmethod(lambda a, b, am, bm: torch.ops.tt_b200.gemm(a, b, bool(am), bool(bm)))
    # routed experts (the padded expert layout needs no host read, so MoE steps trace too)
    router_topk = staticmethod(lambda lg, bias, k, sig, g, lim: torch.ops.tt_b200_graph.router_topk(
        lg, bias, int(k), bool(sig), int(g), int(lim)))
    gather_rows = staticmethod(lambda src, idx: torch.ops.tt_b200_graph.gather_rows(src, idx))
    gemm_grouped_rows = staticmethod(lambda a, b, tg, n, rows, bmn: torch.ops.tt_b200_graph.gemm_grouped_rows(
        a, b, tg, int(n), int(rows), bool(bmn)))
    gemm_grouped_k = staticmethod(lambda a, b, ks, kl: torch.ops.tt_b200_graph.gemm_grouped_k(a, b, ks, kl))
    moe_combine_fwd = staticmethod(lambda base, y, pos, w: torch.ops.tt_b200_graph.moe_combine_fwd(base, y, pos, w))
    moe_combine_bwd = staticmethod(lambda dout, y, pos, tok, scale, need: torch.ops.tt_b200_graph.moe_combine_bwd(
        dout, y, pos, tok, scale, bool(need)))

    @staticmethod
    def attn_fwd(q, k, v, causal, scale, doc_start=None, doc_end=None):
        return torch.ops.tt_b200.attn_fwd(q, k, v, bool(causal), float(scale), doc_start, doc_end)

    @staticmethod
    def attn_bwd(dout, q, k, v, o, lse, causal, scale, dlse=None, doc_start=None, doc_end=None):
        return torch.ops.tt_b200_graph.attn_bwd(dout, q, k, v, o, lse, bool(causal), float(scale), dlse,
                                                doc_start, doc_end)

    def __getattr__(self, name):
        return getattr(_C(), name)


_NS = _TraceableKernels()


@contextlib.contextmanager
def traceable_kernels() -> Iterator[None]:
    prev = _ext._trace_ns
    _ext._trace_ns = _NS
    try:
        yield
    finally:
        _ext._trace_ns = prev
