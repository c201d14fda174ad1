"""Token-choice top-k Mixture of Experts (parity: ``models/common/moe.py:24-489``).

Router: ``gate`` linear -> sigmoid (or softmax) in fp32 -> optional grouped
(node-limited) selection -> top-k on ``scores + expert_bias`` (the bias only
steers selection; gating weights come from the unbiased scores) ->
optional renormalisation and ``route_scale``.  Routed tokens are sorted by
expert, scaled by their gate before the experts (``score_before_experts``),
run through SwiGLU experts with stacked weights ``w1/w3 [E, H, D]`` and
``w2 [E, D, H]``, and summed back per token.

Load balancing: the aux-loss-free expert bias (``expert_bias``, updated by an
optimizer pre-hook from ``tokens_per_expert``) as in the reference, plus an
optional auxiliary loss (``aux_loss_coeff``; absent in the reference)
injected through an identity autograd node so the trainer's loss code is
unchanged: L_aux = coeff * E * sum_e f_e * p_e with f_e the fraction of
routed slots taken by expert e and p_e its mean normalised router score.

Expert parallelism replaces the local expert call with ``ep_dispatch``
(``parallel.expert_parallel``).
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from torchtitan_b200 import ops

from .layers import FeedForward, Linear, _local


class _AuxLossInjector(torch.autograd.Function):
    """Returns x unchanged; backward also feeds d(aux)/d(aux) = 1 into ``aux``."""

    @staticmethod
    def forward(ctx, x, aux):
        ctx.save_for_backward(aux)
        return x

    @staticmethod
    def backward(ctx, g):
        (aux,) = ctx.saved_tensors
        return g, torch.ones_like(aux)


def _router_kernel_enabled() -> bool:
    # csrc/router_topk.cu by default (validated on a B200); TTB_ROUTER_KERNEL=0 selects PyTorch
    import os

    return os.environ.get("TTB_ROUTER_KERNEL", "1") != "0"


class TokenChoiceTopKRouter(nn.Module):
    def __init__(self, dim: int, num_experts: int, top_k: int, score_func: str = "sigmoid",
                 route_norm: bool = False, route_scale: float = 1.0, num_expert_groups: int | None = None,
                 num_limited_groups: int | None = None):
        super().__init__()
        self.gate = Linear(dim, num_experts)
        self.num_experts, self.top_k = num_experts, top_k
        self.score_func, self.route_norm, self.route_scale = score_func, route_norm, route_scale
        self.num_expert_groups, self.num_limited_groups = num_expert_groups, num_limited_groups
        self.force_load_balance = False

    def init_weights(self, std: float) -> None:
        self.gate.init_weights(std)

    def _group_limit(self, s: torch.Tensor) -> torch.Tensor:
        G = self.num_expert_groups
        grouped = s.view(-1, G, self.num_experts // G)
        group_score = grouped.topk(2, dim=-1).values.sum(-1)
        keep = group_score.topk(self.num_limited_groups, dim=-1).indices
        mask = torch.ones_like(group_score, dtype=torch.bool).scatter_(1, keep, False)
        return grouped.masked_fill(mask[..., None], float("-inf")).view(-1, self.num_experts)

    def forward(self, x: torch.Tensor, expert_bias: torch.Tensor | None = None):
        logits = self.gate(x).float()
        scores = torch.sigmoid(logits) if self.score_func == "sigmoid" else F.softmax(logits, dim=-1)
        if logits.is_cuda and not self.force_load_balance and _router_kernel_enabled():
            # selection (bias, group limit, top-k, counts) in one kernel; weights stay in autograd
            from torchtitan_b200.ops._ext import ext

            G = self.num_expert_groups or 1
            idx, counts = ext().router_topk(logits.detach().contiguous(), expert_bias, self.top_k,
                                            self.score_func == "sigmoid", G, self.num_limited_groups or 1)
            top = scores.gather(1, idx)
            if self.route_norm:
                top = top / (top.sum(-1, keepdim=True) + 1e-20)
            return top * self.route_scale, idx, counts.long(), scores
        choice = scores if expert_bias is None else scores + expert_bias.float()
        if self.num_expert_groups is not None and self.num_expert_groups > 1:
            choice = self._group_limit(choice)
        if self.force_load_balance:
            n = x.shape[0]
            idx = (torch.arange(n * self.top_k, device=x.device) % self.num_experts).view(n, self.top_k)
        else:
            idx = choice.topk(self.top_k, dim=-1, sorted=False).indices
        top = scores.gather(1, idx)
        if self.route_norm:
            top = top / (top.sum(-1, keepdim=True) + 1e-20)
        top = top * self.route_scale
        counts = torch.bincount(idx.flatten(), minlength=self.num_experts)
        return top, idx, counts, scores


class _GradScale(torch.autograd.Function):
    @staticmethod
    def forward(ctx, w, s):
        ctx.s = s
        return w.view_as(w)

    @staticmethod
    def backward(ctx, g):
        return g * ctx.s, None


class GroupedExperts(nn.Module):
    grad_scale = 1.0  # set by FSDP on gloo, where expert and dense reductions average over different meshes
    grad_reduce_group = None  # tensor parallelism with sequence-sharded tokens: reduce weight grads over TP

    def __init__(self, dim: int, hidden_dim: int, num_experts: int):
        super().__init__()
        self.num_experts, self.dim, self.hidden_dim = num_experts, dim, hidden_dim
        self.w1 = nn.Parameter(torch.empty(num_experts, hidden_dim, dim))
        self.w2 = nn.Parameter(torch.empty(num_experts, dim, hidden_dim))
        self.w3 = nn.Parameter(torch.empty(num_experts, hidden_dim, dim))

    def init_weights(self, std: float) -> None:
        for w in (self.w1, self.w2, self.w3):
            nn.init.trunc_normal_(w, std=std)

    def forward(self, x: torch.Tensor, counts: torch.Tensor) -> torch.Tensor:
        """x: [sum(counts), D] rows sorted by (local) expert."""
        return ops.grouped_swiglu(x, *self.weights(), counts)

    def weights(self):
        ws = [_local(w) for w in (self.w1, self.w2, self.w3)]
        if self.grad_reduce_group is not None:
            from torchtitan_b200.parallel.tensor_parallel import grad_all_reduce

            ws = [grad_all_reduce(w, self.grad_reduce_group) for w in ws]
        if self.grad_scale != 1.0:
            ws = [_GradScale.apply(w, self.grad_scale) for w in ws]
        return ws


class MoE(nn.Module):
    def __init__(self, dim: int, hidden_dim: int, num_experts: int, top_k: int, *, score_func: str = "sigmoid",
                 route_norm: bool = False, route_scale: float = 1.0, num_expert_groups: int | None = None,
                 num_limited_groups: int | None = None, shared_hidden_dim: int | None = None,
                 load_balance_coeff: float | None = 1e-3, aux_loss_coeff: float = 0.0,
                 score_before_experts: bool = True):
        super().__init__()
        self.num_experts, self.top_k = num_experts, top_k
        self.router = TokenChoiceTopKRouter(dim, num_experts, top_k, score_func, route_norm, route_scale,
                                            num_expert_groups, num_limited_groups)
        self.experts = GroupedExperts(dim, hidden_dim, num_experts)
        self.shared_experts = FeedForward(dim, shared_hidden_dim) if shared_hidden_dim else None
        self.score_before_experts = score_before_experts
        self.load_balance_coeff = load_balance_coeff
        self.aux_loss_coeff = aux_loss_coeff
        if load_balance_coeff is not None:
            self.register_buffer("expert_bias", torch.zeros(num_experts, dtype=torch.float32), persistent=True)
        else:
            self.expert_bias = None
        self.register_buffer("tokens_per_expert", torch.zeros(num_experts, dtype=torch.float32), persistent=False)
        self.last_aux_loss: torch.Tensor | None = None
        self.ep_dispatch = None  # set by expert parallelism

    def init_weights(self, std: float = 0.02) -> None:
        self.router.init_weights(std)
        self.experts.init_weights(std)
        if self.shared_experts is not None:
            self.shared_experts.init_weights(std)
        with torch.no_grad():
            if self.expert_bias is not None:
                self.expert_bias.zero_()
            self.tokens_per_expert.zero_()

    etp_group = None  # expert tensor parallelism: hidden dims of the experts sharded over TP
    etp_sequence_parallel = False

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.etp_group is None:
            return self._forward_core(x)
        from torchtitan_b200.parallel import tensor_parallel as tp

        # every TP rank routes all tokens and computes its slice of every expert's hidden
        # dim; the partial outputs are summed (and re-sharded along the sequence)
        g = self.etp_group
        x = tp.all_gather_seq(x, g) if self.etp_sequence_parallel else tp.grad_all_reduce(x, g)
        out = self._forward_core(x)
        return tp.reduce_scatter_seq(out, g) if self.etp_sequence_parallel else tp.all_reduce(out, g)

    def _forward_core(self, x: torch.Tensor) -> torch.Tensor:
        B, S, D = x.shape
        xf = x.reshape(-1, D)
        top, idx, counts, scores = self.router(xf, self.expert_bias)
        with torch.no_grad():
            self.tokens_per_expert.add_(counts.float())
        flat = idx.flatten()
        order = torch.argsort(flat, stable=True)
        token_of = order // self.top_k
        gates = top.flatten()[order]
        kernels = ops.combine_kernel_enabled(xf)
        if kernels:
            # deterministic gather / gather-sum kernels in both directions (no atomics)
            pos = ops.slot_positions(order, self.top_k)
            routed = ops.moe_dispatch(xf, token_of, pos)
        else:
            routed = xf[token_of]
        if self.score_before_experts:
            routed = (routed.float() * gates[:, None]).to(x.dtype)
        if self.ep_dispatch is not None:
            out_routed = self.ep_dispatch(routed, counts, self.experts)
        else:
            out_routed = self.experts(routed, counts)
        if kernels and out_routed.dtype == torch.bfloat16:
            base = self.shared_experts(x).reshape(-1, D) if self.shared_experts is not None else None
            if base is not None and base.dtype != torch.bfloat16:
                base = base.to(torch.bfloat16)
            w = None if self.score_before_experts else top
            out = ops.moe_combine(base, out_routed, w, pos, token_of, order).to(x.dtype).view(B, S, D)
        else:
            if not self.score_before_experts:
                out_routed = (out_routed.float() * gates[:, None]).to(x.dtype)
            out = self.shared_experts(x).reshape(-1, D) if self.shared_experts is not None else torch.zeros_like(xf)
            out = out.index_add(0, token_of, out_routed.to(out.dtype)).view(B, S, D)
        if self.aux_loss_coeff > 0 and self.training:
            p = scores / (scores.sum(-1, keepdim=True) + 1e-20)
            f = counts.float() / max(flat.numel(), 1)
            aux = self.aux_loss_coeff * self.num_experts * (f.detach() * p.mean(0)).sum()
            self.last_aux_loss = aux.detach()
            out = _AuxLossInjector.apply(out, aux)
        return out
