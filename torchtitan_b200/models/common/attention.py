"""Grouped-query attention block (parity: ``models/common/attention.py:700-746``).

``x -> wq/wk/wv -> RoPE(q,k) -> flash attention -> wo``.  Under tensor
parallelism the projections are column/row parallel and this module sees only
its local heads (derived from the local weight shapes).  Under context
parallelism a ``cp`` hook (``parallel.context_parallel``) wraps the inner
attention: Ulysses all-to-alls sequence<->heads, or ring attention rotates KV.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from torchtitan_b200 import ops

from .layers import Linear, _local


def document_causal_mask(doc_ids: torch.Tensor) -> torch.Tensor:
    """[B,S] document ids -> [B,1,S,S] bool mask (causal within a document)."""
    S = doc_ids.shape[-1]
    causal = torch.ones(S, S, dtype=torch.bool, device=doc_ids.device).tril()
    same = doc_ids[:, :, None] == doc_ids[:, None, :]
    return (causal & same)[:, None]


def _ulysses_fused_enabled() -> bool:
    import os

    return os.environ.get("TTB_ULYSSES_FUSED", "1") != "0"


class GQAttention(nn.Module):
    def __init__(self, dim: int, n_heads: int, n_kv_heads: int | None = None, head_dim: int | None = None,
                 qk_norm: bool = False, norm_eps: float = 1e-5, mask_type: str = "causal"):
        super().__init__()
        self.n_heads = n_heads
        self.n_kv_heads = n_kv_heads or n_heads
        self.head_dim = head_dim or dim // n_heads
        self.wq = Linear(dim, n_heads * self.head_dim)
        self.wk = Linear(dim, self.n_kv_heads * self.head_dim)
        self.wv = Linear(dim, self.n_kv_heads * self.head_dim)
        self.wo = Linear(n_heads * self.head_dim, dim)
        self.mask_type = mask_type
        self.cp_hook = None  # set by context parallelism
        self.kv_cache: dict | None = None  # set by generation (keys/values of earlier positions)
        if qk_norm:
            from .layers import RMSNorm

            self.q_norm = RMSNorm(self.head_dim, norm_eps)
            self.k_norm = RMSNorm(self.head_dim, norm_eps)
        else:
            self.q_norm = self.k_norm = None

    def init_weights(self, init_std: float) -> None:
        for lin in (self.wq, self.wk, self.wv):
            lin.init_weights(0.02)
        self.wo.init_weights(init_std)
        for n in (self.q_norm, self.k_norm):
            if n is not None:
                n.init_weights()

    def inner_attention(self, q, k, v, attention_masks=None):
        if self.mask_type == "block_causal" and attention_masks is not None:
            if q.is_cuda:
                return ops.document_attention(q, k, v, attention_masks)
            from torchtitan_b200.ops import reference as R

            H, Hk = q.shape[2], k.shape[2]
            kk = k.repeat_interleave(H // Hk, 2)
            vv = v.repeat_interleave(H // Hk, 2)
            o = torch.nn.functional.scaled_dot_product_attention(
                q.transpose(1, 2).float(), kk.transpose(1, 2).float(), vv.transpose(1, 2).float(),
                attn_mask=document_causal_mask(attention_masks))
            return o.transpose(1, 2).to(q.dtype)
        return ops.attention(q, k, v, causal=True)

    def forward(self, x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, attention_masks=None) -> torch.Tensor:
        B, S, _ = x.shape
        g = getattr(self, "cp_group", None)
        if (g is not None and attention_masks is None and self.kv_cache is None and self.mask_type == "causal"
                and _ulysses_fused_enabled()):
            from torchtitan_b200.parallel import context_parallel as cpx

            if cpx._ulysses_fused_ok(self, x, g):
                return cpx.ulysses_fused_forward(self, x, cos, sin, g)
        q = self.wq(x)
        k = self.wk(x)
        v = self.wv(x)
        Sq = q.shape[1]
        q = q.view(B, Sq, -1, self.head_dim)
        k = k.view(B, Sq, -1, self.head_dim)
        v = v.view(B, Sq, -1, self.head_dim)
        if self.q_norm is not None:
            q = self.q_norm(q)
            k = self.k_norm(k)
        q = ops.rope(q, cos, sin)
        k = ops.rope(k, cos, sin)
        if self.kv_cache is not None:  # incremental decoding: attend to every cached position too
            if self.kv_cache:
                k = torch.cat([self.kv_cache["k"], k], 1)
                v = torch.cat([self.kv_cache["v"], v], 1)
            self.kv_cache["k"], self.kv_cache["v"] = k, v
        if self.cp_hook is not None:
            o = self.cp_hook(self.inner_attention, q, k, v, attention_masks)
        else:
            o = self.inner_attention(q, k, v, attention_masks)
        return self.wo(o.reshape(B, Sq, -1))
