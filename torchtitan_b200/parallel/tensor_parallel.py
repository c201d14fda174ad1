"""Tensor + sequence parallelism with explicit collectives.

Between TP regions activations are sequence-sharded ``[B, S/tp, D]``.  A
column-parallel linear all-gathers the sequence then multiplies by its local
output-feature shard; a row-parallel linear multiplies its local
input-feature shard and reduce-scatters the partial sums back to sequence
shards (parity of placement: ``models/llama3/parallelize.py:142-241``).
Weights are DTensors on the ``tp`` mesh (``Shard(0)`` col / ``Shard(1)`` row)
so FSDP2 composes on top and DCP reshards them.  Parameters replicated over
TP (norm weights, embeddings) get their gradients all-reduced over TP because
each rank sees a different sequence shard.

``enable_async_tensor_parallel`` switches the column/row linears to the
ring-decomposed collective matmuls of ``parallel.async_tp``: GEMM on the
sequence chunk present overlaps the transfer of the next one.
"""
from __future__ import annotations

from typing import Any

import torch
import torch.distributed as dist
import torch.nn as nn

from torchtitan_b200 import ops


# ------------------------------------------------------------------ collectives
def _all_gather_seq(x: torch.Tensor, group) -> torch.Tensor:
    w = dist.get_world_size(group)
    xs = x.transpose(0, 1).contiguous()  # [S/tp, B, ...]
    out = torch.empty((w * xs.shape[0],) + tuple(xs.shape[1:]), dtype=x.dtype, device=x.device)
    dist.all_gather_into_tensor(out, xs, group=group)
    return out.transpose(0, 1)


def _reduce_scatter_seq(x: torch.Tensor, group) -> torch.Tensor:
    w = dist.get_world_size(group)
    xs = x.transpose(0, 1).contiguous()
    out = torch.empty((xs.shape[0] // w,) + tuple(xs.shape[1:]), dtype=x.dtype, device=x.device)
    dist.reduce_scatter_tensor(out, xs, group=group)
    return out.transpose(0, 1)


class _AGSeq(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return _all_gather_seq(x, group)

    @staticmethod
    def backward(ctx, g):
        return _reduce_scatter_seq(g, ctx.group), None


class _RSSeq(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return _reduce_scatter_seq(x, group)

    @staticmethod
    def backward(ctx, g):
        return _all_gather_seq(g, ctx.group), None


class _AllReduce(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        x = x.clone()
        dist.all_reduce(x, group=group)
        return x

    @staticmethod
    def backward(ctx, g):
        return g, None


class _GradAllReduce(torch.autograd.Function):
    """Identity forward; all-reduce the gradient over ``group`` in backward."""

    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return x.view_as(x)

    @staticmethod
    def backward(ctx, g):
        g = g.contiguous()
        dist.all_reduce(g, group=ctx.group)
        return g, None


def all_gather_seq(x, group):
    return _AGSeq.apply(x, group)


def reduce_scatter_seq(x, group):
    return _RSSeq.apply(x, group)


def all_reduce(x, group):
    """Sum over ``group`` in forward, identity in backward (row-parallel partial sums)."""
    return _AllReduce.apply(x, group)


def grad_all_reduce(x, group):
    return _GradAllReduce.apply(x, group)


def tp_linear(x: torch.Tensor, w: torch.Tensor, mode: str, group, sequence_parallel: bool,
              matmul=None) -> torch.Tensor:
    """``matmul(x, w)`` (default ``ops.linear``; quantized recipes pass their own) with the
    TP collectives around it."""
    mm = matmul or ops.linear
    from . import async_tp

    if async_tp.ENABLED and sequence_parallel and matmul is None and dist.get_world_size(group) > 1:
        if mode == "col":
            return async_tp.ag_matmul(x, w, group)
        if mode == "row":
            return async_tp.matmul_rs(x, w, group)
    if mode == "row_local":
        # partial output summed by the caller together with other partial sums
        return mm(x, w)
    if mode == "col_local":
        # input already complete on every rank and its gradient left partial on purpose: the
        # producer of the input reduces it (see apply_tp_mla)
        return mm(x, w)
    if mode == "col":
        # replicated input: each rank's dgrad is a partial sum over its output shard
        x = all_gather_seq(x, group) if sequence_parallel else grad_all_reduce(x, group)
        return mm(x, w)
    if mode == "row":
        y = mm(x, w)
        return reduce_scatter_seq(y, group) if sequence_parallel else _AllReduce.apply(y, group)
    raise ValueError(mode)


# ------------------------------------------------------------ vocab-parallel CE
def _per_rank(fn):
    """Run ``fn`` once per simulated rank under LocalTensorMode (rank-dependent offsets into a
    plain tensor); unchanged otherwise."""
    try:
        from torch.distributed._local_tensor import maybe_run_for_local_tensor
    except ImportError:
        return fn
    return maybe_run_for_local_tensor(fn)


@_per_rank
def _shift_labels(labels: torch.Tensor, rank: int, vloc: int) -> torch.Tensor:
    return labels - rank * vloc


class _VocabParallelCE(torch.autograd.Function):
    """Sum CE over tokens with logits sharded on the vocab dim across ``group``."""

    @staticmethod
    def forward(ctx, logits, labels, group, ignore_index, rank):
        lf = logits.float()
        ws = dist.get_world_size(group)
        vloc = lf.shape[-1]
        mx = lf.max(-1).values
        dist.all_reduce(mx, op=dist.ReduceOp.MAX, group=group)
        ex = torch.exp(lf - mx[:, None])
        se = ex.sum(-1)
        dist.all_reduce(se, group=group)
        valid = labels != ignore_index
        local_lab = _shift_labels(labels, rank, vloc)
        mine = valid & (local_lab >= 0) & (local_lab < vloc)
        idx = local_lab.clamp(0, vloc - 1)
        tgt = torch.where(mine, lf.gather(1, idx[:, None])[:, 0], 0.0)
        dist.all_reduce(tgt, group=group)
        lse = mx + se.log()
        loss = ((lse - tgt) * valid).sum()
        ctx.save_for_backward(ex, se, idx, mine, valid)
        ctx.dtype = logits.dtype
        return loss

    @staticmethod
    def backward(ctx, g):
        ex, se, idx, mine, valid = ctx.saved_tensors
        p = ex / se[:, None]
        p.scatter_add_(1, idx[:, None], -mine.to(p.dtype)[:, None])
        p *= (valid.float() * g)[:, None]
        return p.to(ctx.dtype), None, None, None, None


def vocab_parallel_cross_entropy_sum(logits, labels, group, ignore_index=-100, rank=None):
    """``rank``: this rank's index in ``group`` (default ``dist.get_rank(group)``; the mesh's
    ``get_local_rank()`` carries the per-rank value when one process simulates every rank)."""
    if rank is None:
        rank = dist.get_rank(group)
    return _VocabParallelCE.apply(logits.flatten(0, -2), labels.flatten(), group, ignore_index, rank)


# ---------------------------------------------------------------- application
def _shard_param(mod: nn.Module, name: str, mesh, placement) -> None:
    from torch.distributed.tensor import distribute_tensor

    p = getattr(mod, name)
    setattr(mod, name, nn.Parameter(distribute_tensor(p.data, mesh, [placement]), requires_grad=p.requires_grad))


def _replicate_param(mod: nn.Module, name: str, mesh) -> None:
    from torch.distributed.tensor import Replicate, distribute_tensor

    p = getattr(mod, name)
    setattr(mod, name, nn.Parameter(distribute_tensor(p.data, mesh, [Replicate()]), requires_grad=p.requires_grad))


def parallelize_linear(lin: nn.Module, mode: str, tp_mesh, sequence_parallel: bool) -> None:
    from torch.distributed.tensor import Shard

    _shard_param(lin, "weight", tp_mesh, Shard(1 if mode in ("row", "row_local") else 0))
    if getattr(lin, "bias", None) is not None:
        if mode in ("col", "col_local"):
            _shard_param(lin, "bias", tp_mesh, Shard(0))
        elif sequence_parallel:  # added after the reduce-scatter: each rank sees its own tokens
            lin.bias_grad_reduce_group = tp_mesh.get_group()
    lin.tp_mode = mode
    lin.tp_group = tp_mesh.get_group()
    lin.sequence_parallel = sequence_parallel


class _TPNorm(nn.Module):
    """Wraps a replicated-over-TP norm so its weight grad is all-reduced."""


def wrap_replicated_norm(norm: nn.Module, tp_mesh) -> None:
    _replicate_param(norm, "weight", tp_mesh)
    group = tp_mesh.get_group()
    orig = norm.forward

    def fwd(x, _orig=orig, _norm=norm):
        from torchtitan_b200 import ops as _ops

        w = _norm.weight.to_local()
        w = grad_all_reduce(w, group)
        return _ops.rms_norm(x, w.to(x.dtype), _norm.eps)

    norm.forward = fwd


@_per_rank
def _seq_shard(tokens: torch.Tensor, r: int, ws: int) -> torch.Tensor:
    S = tokens.shape[1]
    return tokens[:, r * S // ws:(r + 1) * S // ws]


def _tp_embed_and_head(model: nn.Module, tp_mesh, loss_parallel: bool, sequence_parallel: bool) -> None:
    """Embedding replicated (embeds the local sequence shard under SP), final norm
    sequence-parallel, output head column-parallel over the vocabulary."""
    group = tp_mesh.get_group()
    ws = tp_mesh.size()
    if sequence_parallel and model.norm is not None:
        wrap_replicated_norm(model.norm, tp_mesh)
    if model.tok_embeddings is not None:
        _replicate_param(model.tok_embeddings, "weight", tp_mesh)
        emb = model.tok_embeddings

        def emb_fwd(tokens, _emb=emb):
            w = grad_all_reduce(_emb.weight.to_local(), group) if sequence_parallel else _emb.weight.to_local()
            if sequence_parallel:
                r = tp_mesh.get_local_rank()  # per rank under LocalTensorMode too
                tokens = _seq_shard(tokens, r, ws)
            return nn.functional.embedding(tokens, w)

        emb.forward = emb_fwd
    if model.output is not None:
        parallelize_linear(model.output, "col", tp_mesh, sequence_parallel)
        model.output.loss_parallel = loss_parallel
        if not loss_parallel:
            orig = model.output.forward

            def out_fwd(x, _orig=orig):
                y = _orig(x)
                outs = [torch.empty_like(y) for _ in range(ws)]
                dist.all_gather(outs, y.contiguous(), group=group)
                return torch.cat(outs, -1)

            model.output.forward = out_fwd
    model._tp_group = group
    model._tp_rank = tp_mesh.get_local_rank()
    model._tp_loss_parallel = loss_parallel
    model._sp_degree = ws if sequence_parallel else 1


def apply_tp_llama(model: nn.Module, tp_mesh, *, loss_parallel: bool, sequence_parallel: bool = True) -> None:
    """TP plan for dense decoders: q/k/v/w1/w3 column, wo/w2 row, norms
    sequence-parallel, embedding replicated (embeds the local sequence shard),
    output column-parallel (vocab shards, loss parallel)."""
    group = tp_mesh.get_group()
    ws = tp_mesh.size()
    for blk in model.layers.values():
        att = blk.attention
        if hasattr(att, "wkv_a"):  # multi-head latent attention
            apply_tp_mla(att, tp_mesh, sequence_parallel)
            for n in (blk.attention_norm, blk.ffn_norm) if sequence_parallel else ():
                wrap_replicated_norm(n, tp_mesh)
            ff = getattr(blk, "feed_forward", None)
            if ff is not None:
                parallelize_linear(ff.w1, "col", tp_mesh, sequence_parallel)
                parallelize_linear(ff.w3, "col", tp_mesh, sequence_parallel)
                parallelize_linear(ff.w2, "row", tp_mesh, sequence_parallel)
            continue
        if att.n_kv_heads % ws or att.n_heads % ws:
            raise ValueError(f"TP degree {ws} must divide n_heads {att.n_heads} and n_kv_heads {att.n_kv_heads}")
        for lin in (att.wq, att.wk, att.wv):
            parallelize_linear(lin, "col", tp_mesh, sequence_parallel)
        parallelize_linear(att.wo, "row", tp_mesh, sequence_parallel)
        for n in (getattr(att, "q_norm", None), getattr(att, "k_norm", None)):
            if n is not None:  # per-head norms see only this rank's heads: reduce their weight grads
                wrap_replicated_norm(n, tp_mesh)
        ff = getattr(blk, "feed_forward", None)  # MoE blocks: experts are handled by the caller
        if ff is not None:
            parallelize_linear(ff.w1, "col", tp_mesh, sequence_parallel)
            parallelize_linear(ff.w3, "col", tp_mesh, sequence_parallel)
            parallelize_linear(ff.w2, "row", tp_mesh, sequence_parallel)
        if sequence_parallel:
            wrap_replicated_norm(blk.attention_norm, tp_mesh)
            wrap_replicated_norm(blk.ffn_norm, tp_mesh)
    _tp_embed_and_head(model, tp_mesh, loss_parallel, sequence_parallel)


def apply_tp_gpt_oss(model: nn.Module, tp_mesh, *, loss_parallel: bool, sequence_parallel: bool,
                     etp: bool = False) -> None:
    """GPT-OSS: q/k/v column-parallel (weights and biases), o row-parallel, sinks sharded
    with their heads; the MoE (router, experts with biases) is replicated over TP and, on
    sequence shards, its gradients are summed over TP.  With ``etp`` the experts shard their
    hidden dim instead (mlp1 weight and bias along the interleaved gate/up rows, mlp2 along its
    input), the MoE block gathers its input and reduces its output once, and the replicated
    output bias is added by TP rank 0 only."""
    from torch.distributed.tensor import Shard

    group = tp_mesh.get_group()
    ws = tp_mesh.size()
    for blk in model.layers.values():
        att = blk.attention
        if att.sinks.shape[0] % ws or att.wk.out_features // att.head_dim % ws:
            raise ValueError(f"TP degree {ws} must divide the query and key/value head counts")
        for lin in (att.wq, att.wk, att.wv):
            parallelize_linear(lin, "col", tp_mesh, sequence_parallel)
        parallelize_linear(att.wo, "row", tp_mesh, sequence_parallel)
        _shard_param(att, "sinks", tp_mesh, Shard(0))
        if sequence_parallel:
            wrap_replicated_norm(blk.attention_norm, tp_mesh)
            wrap_replicated_norm(blk.ffn_norm, tp_mesh)
        if etp:
            ex = blk.moe.experts
            if ex.mlp2_weight.shape[2] % ws:
                raise ValueError(f"expert TP degree {ws} must divide the expert hidden dim")
            _shard_param(ex, "mlp1_weight", tp_mesh, Shard(1))
            _shard_param(ex, "mlp1_bias", tp_mesh, Shard(1))
            _shard_param(ex, "mlp2_weight", tp_mesh, Shard(2))
            ex.etp_group = group
            blk.moe.etp_group, blk.moe.etp_sequence_parallel = group, sequence_parallel
            blk.moe.router.gate.grad_reduce_group = group  # partial over the hidden slices
        elif sequence_parallel:
            blk.moe.router.gate.grad_reduce_group = group
            blk.moe.experts.grad_reduce_group = group
    _tp_embed_and_head(model, tp_mesh, loss_parallel, sequence_parallel)


def apply_etp(moe: nn.Module, tp_mesh, sequence_parallel: bool, distribute_experts: bool = True) -> None:
    """Expert tensor parallelism on the TP mesh (parity: reference ``ExpertTensorParallel``,
    ``distributed/expert_parallel.py:232-340``, with etp = tp): routed experts shard their
    hidden dim (w1/w3 ``Shard(1)``, w2 ``Shard(2)``), shared experts are column/row split
    without their own collectives, the router is replicated (its weight gradient, a partial
    sum over the hidden slices, is reduced over TP); the MoE block gathers its input and
    reduces its output once (``MoE.etp_group``).  With expert parallelism as well
    (``distribute_experts=False``), ``apply_ep`` shards the experts over ``[ep, etp]`` in one go."""
    from torch.distributed.tensor import Shard, distribute_tensor

    group = tp_mesh.get_group()
    ex = moe.experts
    for name, dim in ((("w1", 1), ("w3", 1), ("w2", 2)) if distribute_experts else ()):
        p = getattr(ex, name)
        setattr(ex, name, nn.Parameter(distribute_tensor(p.data, tp_mesh, [Shard(dim)])))
    if moe.shared_experts is not None:
        parallelize_linear(moe.shared_experts.w1, "col_local", tp_mesh, False)
        parallelize_linear(moe.shared_experts.w3, "col_local", tp_mesh, False)
        parallelize_linear(moe.shared_experts.w2, "row_local", tp_mesh, False)
    moe.router.gate.grad_reduce_group = group
    moe.etp_group = group
    moe.etp_sequence_parallel = sequence_parallel


def apply_tp_mla(att: nn.Module, tp_mesh, sequence_parallel: bool) -> None:
    """Multi-head latent attention (DeepSeek-V3): head projections ``wq``/``wq_b``/``wkv_b``
    column-parallel and ``wo`` row-parallel; the latent projections ``wq_a``/``wkv_a`` keep
    their full weight but take the column-parallel input path (sequence all-gather, or a
    gradient all-reduce of a replicated input) so every rank sees the whole latent; their
    weight gradients and those of the latent norms -- partial sums over this rank's heads --
    are reduced over TP."""
    ws = tp_mesh.size()
    if att.n_heads % ws:
        raise ValueError(f"TP degree {ws} must divide n_heads {att.n_heads}")
    group = tp_mesh.get_group()
    if att.q_lora_rank == 0:
        parallelize_linear(att.wq, "col", tp_mesh, sequence_parallel)
    else:
        parallelize_linear(att.wq_b, "col_local", tp_mesh, sequence_parallel)
    # wkv_b reads the gathered latent; its input gradient stays partial (as does that of the
    # shared rope key, used by this rank's heads only) and wkv_a reduces both together
    parallelize_linear(att.wkv_b, "col_local", tp_mesh, sequence_parallel)
    parallelize_linear(att.wo, "row", tp_mesh, sequence_parallel)
    latent = [att.wkv_a] + ([att.wq_a] if att.q_lora_rank else [])
    for lin in latent:
        lin.tp_mode, lin.tp_group, lin.sequence_parallel = "col", group, sequence_parallel
        lin.grad_reduce_group = group
    for n in [att.kv_norm] + ([att.q_norm] if att.q_lora_rank else []):
        wrap_replicated_norm(n, tp_mesh)


def apply_tp_kimi(model: nn.Module, tp_mesh, *, loss_parallel: bool) -> None:
    """Kimi-Linear TP plan (parity: reference ``kimi_linear/parallelize.py:73-259``): MLA
    heads (``q_proj``, ``kv_b_proj`` column, ``o_proj`` row) and dense MLPs are sharded;
    KDA layers, the latent projection, norms and routed experts are computed replicated
    on every TP rank (activations are replicated, no sequence parallelism); the LM head
    is column-parallel over the vocabulary (loss parallel)."""
    group = tp_mesh.get_group()
    ws = tp_mesh.size()
    for blk in model.layers.values():
        att = blk.self_attn
        if not blk.is_linear_attn:
            if att.h % ws:
                raise ValueError(f"TP degree {ws} must divide num_attention_heads {att.h}")
            parallelize_linear(att.q_proj, "col", tp_mesh, False)
            parallelize_linear(att.kv_b_proj, "col", tp_mesh, False)
            parallelize_linear(att.o_proj, "row", tp_mesh, False)
            att.tp_group = group
        if not blk.is_moe:
            parallelize_linear(blk.ffn.gate_proj, "col", tp_mesh, False)
            parallelize_linear(blk.ffn.up_proj, "col", tp_mesh, False)
            parallelize_linear(blk.ffn.down_proj, "row", tp_mesh, False)
    if model.lm_head is not None:
        parallelize_linear(model.lm_head, "col", tp_mesh, False)
        if not loss_parallel:
            orig = model.lm_head.forward

            def out_fwd(x, _orig=orig):
                y = _orig(x)
                outs = [torch.empty_like(y) for _ in range(ws)]
                dist.all_gather(outs, y.contiguous(), group=group)
                return torch.cat(outs, -1)

            model.lm_head.forward = out_fwd
    model._tp_group = group
    model._tp_rank = tp_mesh.get_local_rank()
    model._tp_loss_parallel = loss_parallel
    model._sp_degree = 1


def maybe_enable_async_tp(parallelism: Any, tp_mesh) -> None:
    """Async TP = ring-decomposed AG->GEMM / GEMM->RS inside the TP linears (no compiler needed)."""
    from . import async_tp

    async_tp.ENABLED = bool(parallelism.enable_async_tensor_parallel)
