"""GPT-OSS (parity: reference ``models/gpt_oss/``, ``moe.py:129-228``).

* Attention: GQA with biases on q/k/v/o, head_dim 64, YaRN RoPE, a learned
  per-head **sink** logit that joins every softmax row (probability mass that
  goes nowhere), and a sliding window of ``sliding_window`` tokens on every
  other layer (even layer indices).
* MoE: router with bias; top-k on the logits, softmax over the selected k;
  experts carry biases and use the clamped SwiGLU
  ``(clamp(up, -L, L) + 1) * g * sigmoid(alpha * g)``, ``g = clamp(gate, max=L)``,
  with gate/up interleaved in one ``mlp1`` projection.

Full-attention layers run on the tcgen05 flash kernel: the sink only rescales
each row by ``sigmoid(lse - sink)`` (differentiable through the kernel's LSE
output).  Sliding-window layers (and CPU) use the PyTorch formulation, O(S^2)
memory per head.
"""
from __future__ import annotations

import dataclasses
import math
from typing import Any

import torch
import torch.nn as nn
import torch.nn.functional as F

from torchtitan_b200 import ops
from torchtitan_b200.protocols import BaseModelArgs
from ..common import Decoder, Embedding, Linear, RMSNorm, RotaryEmbedding
from ..common.blocks import DecoderBlock, init_decoder, nparams_and_flops
from ..common.layers import _local


@dataclasses.dataclass(kw_only=True)
class GptOssModelArgs(BaseModelArgs):
    vocab_size: int = 201088
    dim: int = 2880
    n_layers: int = 24
    n_heads: int = 64
    n_kv_heads: int = 8
    head_dim: int = 64
    norm_eps: float = 1e-5
    num_experts: int = 32
    top_k: int = 4
    moe_inter_dim: int = 2880
    swiglu_limit: float = 7.0
    swiglu_alpha: float = 1.702
    sliding_window: int = 128
    max_seq_len: int = 131072
    original_seq_len: int = 4096
    rope_theta: float = 150000.0
    rope_factor: float = 32.0

    def update_from_config(self, trainer_config: Any) -> None:
        self.max_seq_len = max(self.max_seq_len, trainer_config.training.seq_len)

    def build(self) -> "GptOssModel":
        return GptOssModel(self)

    def get_nparams_and_flops(self, model: nn.Module, seq_len: int) -> tuple[int, float]:
        n, f = nparams_and_flops(model, self.n_layers, self.n_heads, 2 * self.head_dim, seq_len)
        ex = sum(p.numel() for m in model.modules() if isinstance(m, GptOssExperts) for p in m.parameters())
        return n, f - 6 * (ex - ex * self.top_k // self.num_experts)


def sink_attention(q, k, v, sinks, window: int, scale: float):
    """softmax over [q.k scores (causal, optional window) ; sink] then P @ V. q: [B,S,H,D]."""
    B, S, H, D = q.shape
    rep = H // k.shape[2]
    kk = k.repeat_interleave(rep, 2) if rep > 1 else k
    vv = v.repeat_interleave(rep, 2) if rep > 1 else v
    s = torch.einsum("bshd,bthd->bhst", q.float(), kk.float()) * scale
    i = torch.arange(S, device=q.device)
    keep = i[:, None] >= i[None, :]
    if window:
        keep = keep & (i[:, None] - i[None, :] < window)
    s = s.masked_fill(~keep, float("-inf"))
    sink = sinks.float().view(1, H, 1, 1).expand(B, H, S, 1)
    p = torch.softmax(torch.cat([s, sink], -1), -1)[..., :S]
    return torch.einsum("bhst,bthd->bshd", p, vv.float()).to(q.dtype)


def sliding_window_attention_lse(q, k, v, window: int, scale: float):
    """Causal attention limited to the last ``window`` keys (key j visible to query i when
    i - window < j <= i) as two plain causal attentions per window-sized chunk, so the flash
    kernel does the work in O(S * window):

    * chunk c against itself: causal, every key within the window;
    * chunk c against chunk c - 1: local query a sees local key b when b > a.  Reversing both
      orders turns that into "b' < a'", i.e. causal with keys shifted by one: reversed queries
      1..W-1 against reversed keys 0..W-2 (query a = W-1 sees no earlier key and is left out).

    The two partial results merge through their log-sum-exps.  Returns (o, lse) like
    ``ops.attention_with_lse``; q: [B, S, H, D], k/v: [B, S, Hk, D]."""
    B, S, H, D = q.shape
    W = window
    pad = (-S) % W
    F_ = torch.nn.functional
    if pad:  # padded positions come after every real one: causal masking hides them
        q, k, v = (F_.pad(t, (0, 0, 0, 0, 0, pad)) for t in (q, k, v))
    NC = (S + pad) // W

    def chunks(t):  # [B, NC*W, h, d] -> [B*NC, W, h, d]
        return t.reshape(B * NC, W, *t.shape[2:])

    qc, kc, vc = chunks(q), chunks(k), chunks(v)
    o1, l1 = ops.attention_with_lse(qc, kc, vc, causal=True, scale=scale)
    if NC > 1 and W > 1:
        qp = q.reshape(B, NC, W, H, D)[:, 1:].flip(2)[:, :, 1:]                    # reversed queries 1..W-1
        kp = k.reshape(B, NC, W, *k.shape[2:])[:, :-1].flip(2)[:, :, :-1]         # previous chunk, reversed 0..W-2
        vp = v.reshape(B, NC, W, *v.shape[2:])[:, :-1].flip(2)[:, :, :-1]
        o2, l2 = ops.attention_with_lse(qp.reshape(B * (NC - 1), W - 1, H, D).contiguous(),
                                        kp.reshape(B * (NC - 1), W - 1, *k.shape[2:]).contiguous(),
                                        vp.reshape(B * (NC - 1), W - 1, *v.shape[2:]).contiguous(),
                                        causal=True, scale=scale)
        # back to forward order: local queries 0..W-2 of chunks 1..NC-1; the rest see no earlier chunk
        o2 = o2.view(B, NC - 1, W - 1, H, -1).flip(2)
        l2 = l2.view(B, NC - 1, W - 1, H).flip(2)
        neg = torch.full((B, NC, W, H), float("-inf"), device=q.device, dtype=l2.dtype)
        lb = torch.cat([neg[:, :1], torch.cat([l2, neg[:, 1:, :1]], 2)], 1)
        ob = torch.cat([torch.zeros_like(o2[:, :1]).expand(B, 1, W - 1, H, o2.shape[-1]),
                        o2], 1)
        ob = torch.cat([ob, torch.zeros_like(ob[:, :, :1])], 2)
        la = l1.view(B, NC, W, H)
        lse = torch.logaddexp(la, lb)
        oa = o1.view(B, NC, W, H, -1).float()
        o = oa * torch.exp(la - lse)[..., None] + ob.float() * torch.exp(lb - lse)[..., None]
        o, lse = o.reshape(B, NC * W, H, -1), lse.reshape(B, NC * W, H)
    else:
        o, lse = o1.view(B, NC * W, H, -1).float(), l1.view(B, NC * W, H)
    return o[:, :S].to(v.dtype), lse[:, :S]


def _chunked_window_enabled(q: torch.Tensor) -> bool:
    import os

    # default everywhere; TTB_SWA_CHUNKED=0 selects the masked-softmax reference on a GPU
    return not q.is_cuda or os.environ.get("TTB_SWA_CHUNKED", "1") != "0"


class GptOssAttention(nn.Module):
    def __init__(self, a: GptOssModelArgs, layer_id: int):
        super().__init__()
        self.head_dim = a.head_dim
        self.wq = Linear(a.dim, a.n_heads * a.head_dim, bias=True)
        self.wk = Linear(a.dim, a.n_kv_heads * a.head_dim, bias=True)
        self.wv = Linear(a.dim, a.n_kv_heads * a.head_dim, bias=True)
        self.wo = Linear(a.n_heads * a.head_dim, a.dim, bias=True)
        self.sinks = nn.Parameter(torch.empty(a.n_heads))
        self.window = a.sliding_window if layer_id % 2 == 0 else 0
        self.scale = a.head_dim ** -0.5
        if a.max_seq_len > a.original_seq_len:  # YaRN attention factor, applied to q and k (squared)
            self.scale *= (0.1 * math.log(a.rope_factor) + 1.0) ** 2
        self.cp_hook = None

    def init_weights(self, init_std: float) -> None:
        for lin in (self.wq, self.wk, self.wv):
            lin.init_weights(0.02)
        self.wo.init_weights(init_std)
        nn.init.trunc_normal_(self.sinks, std=init_std)

    def inner_attention(self, q, k, v, attention_masks=None):
        if q.is_cuda and not self.window:
            # full layers on the flash kernel: a sink logit s only rescales each row by
            # sum exp / (sum exp + exp s) = sigmoid(lse - s)
            o, lse = ops.attention_with_lse(q, k, v, causal=True, scale=self.scale)
            w = torch.sigmoid(lse - _local(self.sinks).float().view(1, 1, -1))
            return (o.float() * w[..., None]).to(o.dtype)
        if self.window and q.shape[1] > self.window and _chunked_window_enabled(q):
            o, lse = sliding_window_attention_lse(q, k, v, self.window, self.scale)
            w = torch.sigmoid(lse - _local(self.sinks).float().view(1, 1, -1))
            return (o.float() * w[..., None]).to(q.dtype)
        return sink_attention(q, k, v, _local(self.sinks), self.window, self.scale)

    def forward(self, x, cos, sin, attention_masks=None):
        B = x.shape[0]
        q, k, v = self.wq(x), self.wk(x), self.wv(x)
        S = q.shape[1]  # the full sequence under sequence parallelism (the projections gather it)
        q = ops.rope(q.view(B, S, -1, self.head_dim), cos, sin)
        k = ops.rope(k.view(B, S, -1, self.head_dim), cos, sin)
        v = v.view(B, S, -1, self.head_dim)
        if self.cp_hook is not None:
            if self.window:
                raise NotImplementedError("context parallelism with sliding-window layers is not wired")
            o = self.cp_hook(self.inner_attention, q, k, v, attention_masks)
        else:
            o = self.inner_attention(q, k, v, attention_masks)
        return self.wo(o.reshape(B, S, -1))


class GptOssExperts(nn.Module):
    def __init__(self, dim: int, inter: int, num_experts: int, limit: float, alpha: float):
        super().__init__()
        self.num_experts, self.limit, self.alpha = num_experts, limit, alpha
        self.mlp1_weight = nn.Parameter(torch.empty(num_experts, 2 * inter, dim))
        self.mlp1_bias = nn.Parameter(torch.empty(num_experts, 2 * inter))
        self.mlp2_weight = nn.Parameter(torch.empty(num_experts, dim, inter))
        self.mlp2_bias = nn.Parameter(torch.empty(num_experts, dim))

    def init_weights(self, std: float) -> None:
        nn.init.trunc_normal_(self.mlp1_weight, std=0.02)
        nn.init.trunc_normal_(self.mlp2_weight, std=std)
        nn.init.zeros_(self.mlp1_bias)
        nn.init.zeros_(self.mlp2_bias)

    def _act(self, h: torch.Tensor) -> torch.Tensor:
        g, u = h[..., ::2], h[..., 1::2]
        g = g.clamp(max=self.limit)
        u = u.clamp(-self.limit, self.limit)
        return (u + 1) * g * torch.sigmoid(self.alpha * g)

    grad_reduce_group = None  # replicated over TP on sequence-sharded tokens: reduce weight grads
    etp_group = None  # expert tensor parallelism: hidden dims sharded, output bias added by TP rank 0

    def forward(self, x: torch.Tensor, counts: list[int]) -> torch.Tensor:
        w1, b1, w2, b2 = (_local(t) for t in (self.mlp1_weight, self.mlp1_bias, self.mlp2_weight, self.mlp2_bias))
        if self.grad_reduce_group is not None:
            from torchtitan_b200.parallel.tensor_parallel import grad_all_reduce

            w1, b1, w2, b2 = (grad_all_reduce(t, self.grad_reduce_group) for t in (w1, b1, w2, b2))
        if self.etp_group is not None:
            import torch.distributed as dist

            from torchtitan_b200.parallel.tensor_parallel import grad_all_reduce

            # the partial outputs are summed over TP: the (replicated) output bias counts once
            b2 = grad_all_reduce(b2, self.etp_group) * float(dist.get_rank(self.etp_group) == 0)
        outs, start = [], 0
        for e, n in enumerate(counts):
            if n:
                xe = x[start:start + n]
                h = ops.linear(xe, w1[e].to(x.dtype)) + b1[e].to(x.dtype)
                outs.append(ops.linear(self._act(h), w2[e].to(x.dtype)) + b2[e].to(x.dtype))
            start += n
        return torch.cat(outs) if outs else x.new_zeros(0, w2.shape[1])


class GptOssMoE(nn.Module):
    def __init__(self, a: GptOssModelArgs):
        super().__init__()
        self.num_experts, self.top_k = a.num_experts, a.top_k
        self.router = nn.Module()
        self.router.gate = Linear(a.dim, a.num_experts, bias=True)
        self.experts = GptOssExperts(a.dim, a.moe_inter_dim, a.num_experts, a.swiglu_limit, a.swiglu_alpha)
        self.register_buffer("tokens_per_expert", torch.zeros(a.num_experts), persistent=False)

    def init_weights(self, std: float) -> None:
        self.router.gate.init_weights(0.02)
        self.experts.init_weights(std)

    etp_group = None  # expert tensor parallelism (see GptOssExperts)
    etp_sequence_parallel = False

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.etp_group is None:
            return self._forward_core(x)
        from torchtitan_b200.parallel import tensor_parallel as tp

        g = self.etp_group
        x = tp.all_gather_seq(x, g) if self.etp_sequence_parallel else tp.grad_all_reduce(x, g)
        out = self._forward_core(x)
        return tp.reduce_scatter_seq(out, g) if self.etp_sequence_parallel else tp.all_reduce(out, g)

    def _forward_core(self, x: torch.Tensor) -> torch.Tensor:
        B, S, D = x.shape
        xf = x.reshape(-1, D)
        logits = self.router.gate(xf).float()
        top, idx = logits.topk(self.top_k, dim=-1)
        gates = F.softmax(top, dim=-1)
        flat = idx.flatten()
        counts = torch.bincount(flat, minlength=self.num_experts)
        with torch.no_grad():
            self.tokens_per_expert.add_(counts.float())
        order = torch.argsort(flat, stable=True)
        token_of = order // self.top_k
        y = self.experts(xf[token_of], counts.tolist())
        y = y.float() * gates.flatten()[order][:, None]
        return torch.zeros_like(xf, dtype=torch.float32).index_add(0, token_of, y).to(x.dtype).view(B, S, D)


class GptOssModel(Decoder):
    def __init__(self, a: GptOssModelArgs):
        super().__init__()
        self.model_args = a
        self.tok_embeddings = Embedding(a.vocab_size, a.dim)
        scaling = "yarn" if a.max_seq_len > a.original_seq_len else None
        self.rope = RotaryEmbedding(a.head_dim, a.max_seq_len, a.rope_theta, scaling, a.rope_factor,
                                    a.original_seq_len, yarn_truncate=False)
        self.layers = nn.ModuleDict({
            str(i): DecoderBlock(i, a.dim, GptOssAttention(a, i), a.norm_eps, moe=GptOssMoE(a),
                                 init_std=0.02 / (2 * (i + 1)) ** 0.5)
            for i in range(a.n_layers)})
        self.norm = RMSNorm(a.dim, a.norm_eps)
        self.output = Linear(a.dim, a.vocab_size)

    def init_weights(self, buffer_device=None) -> None:
        init_decoder(self, self.model_args.dim, buffer_device)
