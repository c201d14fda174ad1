"""Kimi Delta Attention (KDA): gated delta rule with per-channel decay.

Recurrence for one head (state S in R^{K x V}, per-channel log decay g_t <= 0):

    S'_t = diag(exp(g_t)) S_{t-1}
    S_t  = S'_t + beta_t k_t (v_t - S'_t^T k_t)^T
    o_t  = S_t^T q_t                      (q scaled by 1/sqrt(K), q/k L2-normalised)

``chunk_kda`` evaluates it chunk-parallel (chunk C = 64) in the WY form of
the delta rule (Yang et al., "Parallelizing Linear Transformers with the
Delta Rule over Sequence Length", 2024), with G = within-chunk cumulative
log decay:

    A_kk[i,j] = beta_i sum_d k_i k_j exp(G_i - G_j)        (j < i)
    T         = (I + A_kk)^{-1} diag(beta)
    w = T (exp(G) * k),   u = T v
    per chunk: v' = u - w S;  o = (q * exp(G)) S + A_qk v'   (A_qk: j <= i)
               S <- diag(exp(G_C)) S + (exp(G_C - G) * k)^T v'

Pairwise decayed products are formed per column j with exp(G_i - G_j) <= 1
(never the overflow-prone factorisation exp(G_i) exp(-G_j)); the custom
backward recomputes them instead of saving C x C x K tensors.
Reference semantics: ``fla/ops/kda/naive.py`` (naive_recurrent_kda).
"""
from __future__ import annotations

import os

import torch
import torch.nn.functional as F


def _use_gram_kernel(t: torch.Tensor) -> bool:
    # csrc/kda_gram.cu and csrc/kda_scan.cu on CUDA (TTB_KDA_KERNEL=0 selects the PyTorch loops)
    import os

    return t.is_cuda and os.environ.get("TTB_KDA_KERNEL", "1") != "0"


def _fits_shared_memory(C: int, K: int, V: int = 0) -> bool:
    """The kernels keep per-chunk tiles in shared memory (227 KB per CTA)."""
    gram = 4 * (6 * C * (K + 1) + C * (C + 1))  # backward: tiles, scaled rows, dout, accumulators
    vs = _scan_slice_width(V) if V else 1
    scan = 4 * (2 * K * (vs + 1) + 3 * C * (K + 1) + C * (C + 1) + 3 * C * (vs + 1) + K)
    return max(gram, scan) <= 227 * 1024


class _DecayedGram(torch.autograd.Function):
    """out[n, i, j] = sum_d a[n,i,d] b[n,j,d] exp(G[n,i,d] - G[n,j,d]) for j < i
    (``strict``) or j <= i, else 0.  a, b, G: [N, C, K] fp32.  On CUDA (opt-in)
    one kernel per direction (``csrc/kda_gram.cu``); else a loop over columns."""

    @staticmethod
    def forward(ctx, a, b, G, strict):
        ctx.kernel = _use_gram_kernel(a) and _fits_shared_memory(a.shape[1], a.shape[2])
        if ctx.kernel:
            from ._ext import ext

            a, b, G = (t.float().contiguous() for t in (a, b, G))
            ctx.save_for_backward(a, b, G)
            ctx.strict = strict
            return ext().kda_gram_fwd(a, b, G, strict)
        N, C, K = a.shape
        out = a.new_zeros(N, C, C)
        idx = torch.arange(C, device=a.device)
        for j in range(C):
            e = torch.exp((G - G[:, j : j + 1, :]).clamp(max=0.0))
            col = (a * e * b[:, j : j + 1, :]).sum(-1)  # [N, C]
            keep = (idx > j) if strict else (idx >= j)
            out[:, :, j] = col * keep
        ctx.save_for_backward(a, b, G)
        ctx.strict = strict
        return out

    @staticmethod
    def backward(ctx, dout):
        a, b, G = ctx.saved_tensors
        if ctx.kernel:
            from ._ext import ext

            da, db, dG = ext().kda_gram_bwd(dout.float().contiguous(), a, b, G, ctx.strict)
            return da, db, dG, None
        N, C, K = a.shape
        da, db, dG = torch.zeros_like(a), torch.zeros_like(b), torch.zeros_like(G)
        idx = torch.arange(C, device=a.device)
        for j in range(C):
            keep = (idx > j) if ctx.strict else (idx >= j)
            w = (dout[:, :, j] * keep)[:, :, None]  # [N, C, 1]
            e = torch.exp((G - G[:, j : j + 1, :]).clamp(max=0.0))
            bj = b[:, j : j + 1, :]
            t = w * e  # [N, C, K]
            da += t * bj
            term = t * a  # dO[i,j] a_i e_ij
            db[:, j, :] += term.sum(1)
            full = term * bj
            dG += full
            dG[:, j, :] -= full.sum(1)
        return da, db, dG, None


def decayed_gram(a, b, G, strict: bool):
    return _DecayedGram.apply(a, b, G, strict)


class _Gate(torch.autograd.Function):
    @staticmethod
    def forward(ctx, g_raw, A_log, dt_bias):
        from ._ext import ext

        x = g_raw.contiguous()
        A = A_log.float().reshape(-1).contiguous()
        b = dt_bias.float().reshape(-1).contiguous() if dt_bias is not None else None
        ctx.save_for_backward(x, A, b)
        ctx.shapes = (A_log.shape, A_log.dtype, None if dt_bias is None else (dt_bias.shape, dt_bias.dtype))
        return ext().kda_gate_fwd(x, A, b)

    @staticmethod
    def backward(ctx, dg):
        from ._ext import ext

        x, A, b = ctx.saved_tensors
        dx, dA, db = ext().kda_gate_bwd(x, A, b, dg.float().contiguous())
        (ashape, adtype, bmeta) = ctx.shapes
        dbias = None if bmeta is None else db.reshape(bmeta[0]).to(bmeta[1])
        return dx, dA.reshape(ashape).to(adtype), dbias


def kda_gate(g_raw: torch.Tensor, A_log: torch.Tensor, dt_bias: torch.Tensor | None) -> torch.Tensor:
    """g = -exp(A_log[h]) * softplus(g_raw + dt_bias): [..., H, K] fp32 log decay."""
    if _eltwise_kernels(g_raw) and type(A_log).__name__ != "DTensor" and type(dt_bias).__name__ != "DTensor":
        return _Gate.apply(g_raw, A_log, dt_bias)
    H, K = g_raw.shape[-2:]
    x = g_raw.float()
    if dt_bias is not None:
        x = x + dt_bias.float().view(H, K)
    return -A_log.float().exp().view(H, 1) * F.softplus(x)


def l2norm(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    xf = x.float()
    return xf * torch.rsqrt(xf.pow(2).sum(-1, keepdim=True) + eps)


def _prep_kernel(x: torch.Tensor) -> bool:
    # csrc/kda_prep.cu (TTB_KDA_PREP=0 selects the PyTorch ops)
    return x.is_cuda and os.environ.get("TTB_KDA_PREP", "1") != "0"


class _Prep(torch.autograd.Function):
    """Chunk layout, within-chunk cumulative decay and the decayed q/k operands of every chunk
    in one pass (``csrc/kda_prep.cu``): q, k, g [B, T, H, K] fp32 -> qc, kc, G, exp(G) k,
    exp(G) q, exp(G_last - G) k ([B*H, NT, C, K]) and exp(G_last) ([B*H, NT, K])."""

    @staticmethod
    def forward(ctx, q, k, g, C):
        from ._ext import ext

        outs = ext().kda_prep_fwd(q, k, g, C)
        ctx.save_for_backward(q, k, outs[2])
        ctx.C = C
        return tuple(outs)

    @staticmethod
    def backward(ctx, dqc, dkc, dG, dkg, dqg, dkd, ddecay):
        from ._ext import ext

        q, k, G = ctx.saved_tensors
        c = [None if t is None else t.float().contiguous() for t in (dqc, dkc, dG, dkg, dqg, dkd, ddecay)]
        dq, dk, dg = ext().kda_prep_bwd(q, k, G, ctx.C, *c)
        return dq, dk, dg, None


def chunk_kda(q, k, v, g, beta, scale: float | None = None, chunk_size: int = 64,
              initial_state: torch.Tensor | None = None, output_final_state: bool = False,
              use_qk_l2norm: bool = True):
    """q, k: [B, T, H, K]; v: [B, T, H, V]; g: [B, T, H, K] (log decay, fp32); beta: [B, T, H].

    Returns o [B, T, H, V] (dtype of v) and the final state [B, H, K, V] if requested.
    """
    B, T, H, K = q.shape
    V = v.shape[-1]
    C = chunk_size
    scale = K ** -0.5 if scale is None else scale
    dtype = v.dtype
    if use_qk_l2norm:
        q, k = l2norm(q), l2norm(k)
    q = q.float() * scale
    k, v, g, beta = k.float(), v.float(), g.float(), beta.float()
    pad = (-T) % C
    prep = _prep_kernel(q)
    if pad:
        # padded steps: g = 0 (no decay), k = v = q = 0, beta = 0 -> state unchanged (the prep
        # kernel reads rows past T as zeros itself)
        if not prep:
            q, k, g = (F.pad(x, (0, 0, 0, 0, 0, pad)) for x in (q, k, g))
        v = F.pad(v, (0, 0, 0, 0, 0, pad))
        beta = F.pad(beta, (0, 0, 0, pad))
    Tp = T + pad
    NT = Tp // C

    def chunks(x):  # [B, Tp, H, D] -> [B*H, NT, C, D]
        return x.view(B, NT, C, H, -1).permute(0, 3, 1, 2, 4).reshape(B * H, NT, C, -1)

    bc = beta.view(B, NT, C, H).permute(0, 3, 1, 2).reshape(B * H, NT, C)
    vc = chunks(v)
    N = B * H * NT
    if prep:
        qc, kc, G, kg, qg, kdec, decay = _Prep.apply(q.contiguous(), k.contiguous(), g.contiguous(), C)
    else:
        qc, kc, gc = chunks(q), chunks(k), chunks(g)
        G = gc.cumsum(2)
        kg = G.exp() * kc
        qg = qc * G.exp()
        Glast = G[:, :, -1:, :]  # [BH, NT, 1, K]
        kdec = (Glast - G).exp() * kc
        decay = Glast[:, :, 0, :].exp()  # [BH, NT, K]
    Akk = decayed_gram(kc.reshape(N, C, K), kc.reshape(N, C, K), G.reshape(N, C, K), True).view(B * H, NT, C, C)
    Akk = Akk * bc[..., :, None]
    eye = torch.eye(C, device=q.device, dtype=torch.float32)
    Tm = torch.linalg.solve_triangular(eye + Akk, eye.expand_as(Akk), upper=False, unitriangular=True)
    Tm = Tm * bc[..., None, :]
    w = Tm @ kg
    u = Tm @ vc
    Aqk = decayed_gram(qc.reshape(N, C, K), kc.reshape(N, C, K), G.reshape(N, C, K), False).view(B * H, NT, C, C)
    S0 = None if initial_state is None else initial_state.float().reshape(B * H, K, V)
    o, S = chunk_scan(u, w, qg, Aqk, kdec, decay, S0)
    o = o.view(B, H, NT, C, V).permute(0, 2, 3, 1, 4).reshape(B, Tp, H, V)[:, :T]
    final = S.view(B, H, K, V) if output_final_state else None
    return o.to(dtype), final


def _scan_ref(u, w, qg, Aqk, kdec, decay, S=None):
    """Inter-chunk recurrence as a loop of batched matmuls (any device, autograd through it):
    v' = u - w S;  o = qg S + Aqk v';  S <- diag(decay) S + kdec^T v'."""
    BH, NT, C, V = u.shape
    K = w.shape[-1]
    S = u.new_zeros(BH, K, V) if S is None else S
    outs = []
    for n in range(NT):
        vn = u[:, n] - w[:, n] @ S
        outs.append(qg[:, n] @ S + Aqk[:, n] @ vn)
        S = decay[:, n, :, None] * S + kdec[:, n].transpose(1, 2) @ vn
    return torch.stack(outs, 1), S


def _scan_slice_width(V: int) -> int:
    for vs in (32, 16, 8, 4, 2, 1):
        if V % vs == 0:
            return vs
    return 1


class _ChunkScan(torch.autograd.Function):
    """The recurrence of ``_scan_ref`` from a zero state as one kernel launch per direction
    (``csrc/kda_scan.cu``; grid = V slices x heads, chunk-start states kept for the backward)."""

    @staticmethod
    def forward(ctx, u, w, qg, Aqk, kdec, decay):
        from ._ext import ext

        args = [t.float().contiguous() for t in (u, w, qg, Aqk, kdec, decay)]
        vs = _scan_slice_width(u.shape[-1])
        o, states, fin = ext().kda_scan_fwd(*args, vs)
        ctx.save_for_backward(*args, states)
        ctx.vs = vs
        ctx.set_materialize_grads(False)  # an unused final state brings no gradient (and no sync)
        return o, fin

    @staticmethod
    def backward(ctx, do, dfin):
        from ._ext import ext

        *args, states = ctx.saved_tensors
        if dfin is not None:
            raise NotImplementedError("kda_scan kernel: gradient of the final state is not supported")
        du, dqg, dw, dkd, dA, dd = ext().kda_scan_bwd(do.float().contiguous(), *args, states, ctx.vs)
        return du, dw, dqg, dA, dkd, dd


class _StateScan(torch.autograd.Function):
    """The recurrence of ``_scan_ref`` split the state-passing way: the tcgen05 kernels of
    ``csrc/kda_state.cu`` walk the chunks of each head carrying only the state (forward: S_n and
    v'_n; backward: dS_{n+1} and dv'_n), and everything that does not depend on the walk is a
    batched GEMM over all chunks at once: o = qg S + Aqk v', and the gradients of qg, w, kdec,
    Aqk and the decay.  bf16 operands, fp32 accumulation; the state stays fp32 in TMEM.
    (C = 64 and K = V = 128.)"""

    @staticmethod
    def forward(ctx, u, w, qg, Aqk, kdec, decay, S0):
        from ._ext import ext

        bf = torch.bfloat16
        wb, kdb, qgb, Ab = (t.to(bf).contiguous() for t in (w, kdec, qg, Aqk))
        uT = u.transpose(-1, -2).to(bf).contiguous()
        dec = decay.float().contiguous()
        s0 = None if S0 is None else S0.float().transpose(-1, -2).contiguous()
        states, vnT, fin = ext().kda_state_fwd(wb, kdb, uT, dec, s0)
        # o = qg S_n + Aqk v'_n  (S_n^T and v'^T are what the kernel stored)
        o = torch.matmul(qgb, states.transpose(-1, -2)).float() + torch.matmul(Ab, vnT.transpose(-1, -2)).float()
        ctx.save_for_backward(qgb, wb, kdb, Ab, dec, states, vnT)
        ctx.has_s0 = S0 is not None
        ctx.set_materialize_grads(False)
        return o, fin.transpose(-1, -2)

    @staticmethod
    def backward(ctx, do, dfin):
        from ._ext import ext

        qgb, wb, kdb, Ab, dec, states, vnT = ctx.saved_tensors
        BH, NT, C, K = qgb.shape
        V = states.shape[2]
        dob = (do if do is not None else qgb.new_zeros(BH, NT, C, V)).to(torch.bfloat16).contiguous()
        dfT = None if dfin is None else dfin.float().transpose(-1, -2).contiguous()
        dstates, duT, dS0 = ext().kda_state_bwd(qgb, wb, kdb, dob, Ab, dec, dfT)
        du = duT.transpose(-1, -2)
        dub = du.to(torch.bfloat16)
        # gradients of everything outside the walk, as GEMMs over all chunks
        dqg = torch.matmul(dob, states).float()                                # dO S_n^T
        dw = -torch.matmul(dub, states).float()                                # -dv' S_n^T
        dkdec = torch.matmul(vnT.transpose(-1, -2), dstates).float()           # v' dS_{n+1}^T
        dAqk = torch.matmul(dob, vnT).float()                                  # dO v'^T
        ddec = (dstates.float() * states.float()).sum(-2)                      # sum_v dS_{n+1} o S_n
        dS0 = dS0.transpose(-1, -2) if ctx.has_s0 else None
        return du, dw, dqg, dAqk, dkdec, ddec, dS0


def _state_kernel_ok(u, w) -> bool:
    return (_use_gram_kernel(u) and u.shape[2] == 64 and w.shape[-1] == 128 and u.shape[-1] == 128
            and __import__("os").environ.get("TTB_KDA_STATE", "1") != "0")


def chunk_scan(u, w, qg, Aqk, kdec, decay, S0=None):
    """-> (o [BH, NT, C, V], final state [BH, K, V]); on CUDA the tcgen05 state kernels for
    C = 64, K = V = 128 (``TTB_KDA_STATE=0`` selects the fp32 SIMT recurrence kernels), the SIMT
    kernels for other shapes, and the batched-matmul loop elsewhere."""
    if _state_kernel_ok(u, w):
        return _StateScan.apply(u, w, qg, Aqk, kdec, decay, S0)
    if S0 is None and _use_gram_kernel(u) and _fits_shared_memory(u.shape[2], w.shape[-1], u.shape[-1]):
        return _ChunkScan.apply(u, w, qg, Aqk, kdec, decay)
    return _scan_ref(u, w, qg, Aqk, kdec, decay, S0)


def naive_recurrent_kda(q, k, v, g, beta, scale=None, use_qk_l2norm: bool = True):
    """Token-by-token recurrence (test oracle)."""
    B, T, H, K = q.shape
    V = v.shape[-1]
    scale = K ** -0.5 if scale is None else scale
    if use_qk_l2norm:
        q, k = l2norm(q), l2norm(k)
    q, k, v, g, beta = (x.float() for x in (q, k, v, g, beta))
    q = q * scale
    S = q.new_zeros(B, H, K, V)
    o = torch.zeros(B, T, H, V, dtype=torch.float32, device=q.device)
    for t in range(T):
        S = S * g[:, t, :, :, None].exp()
        kS = (k[:, t, :, :, None] * S).sum(-2)
        S = S + (beta[:, t, :, None] * k[:, t])[..., None] * (v[:, t] - kS)[..., None, :]
        o[:, t] = (q[:, t, :, :, None] * S).sum(-2)
    return o, S


def _eltwise_kernels(x: torch.Tensor) -> bool:
    # csrc/kda_eltwise.cu by default on CUDA; TTB_KDA_ELTWISE=0 selects the PyTorch formulation.
    # Its weight gradients are summed with fp32 atomics (order varies run to run), so under
    # torch.use_deterministic_algorithms the PyTorch formulation runs instead.
    import os

    return (x.is_cuda and x.dtype == torch.bfloat16 and os.environ.get("TTB_KDA_ELTWISE", "1") != "0"
            and not torch.are_deterministic_algorithms_enabled())


class _ShortConv(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight):
        from ._ext import ext

        x = x.contiguous()
        w = weight.float().reshape(weight.shape[0], -1).contiguous()
        ctx.save_for_backward(x, w)
        ctx.wshape, ctx.wdtype = weight.shape, weight.dtype
        return ext().kda_short_conv_fwd(x, w)

    @staticmethod
    def backward(ctx, dy):
        from ._ext import ext

        x, w = ctx.saved_tensors
        dx, dw = ext().kda_short_conv_bwd(x, w, dy.contiguous())
        return dx, dw.reshape(ctx.wshape).to(ctx.wdtype)


class _GatedNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, gate, weight, eps):
        from ._ext import ext

        x, gate = x.contiguous(), gate.to(x.dtype).contiguous()
        g = weight.float().contiguous()
        ctx.save_for_backward(x, gate, g)
        ctx.eps, ctx.wdtype, ctx.gdtype = eps, weight.dtype, gate.dtype
        return ext().kda_gated_norm_fwd(x, gate, g, eps)

    @staticmethod
    def backward(ctx, dy):
        from ._ext import ext

        x, gate, g = ctx.saved_tensors
        dx, dz, dg = ext().kda_gated_norm_bwd(x, gate, g, dy.contiguous(), ctx.eps)
        return dx, dz.to(ctx.gdtype), dg.to(ctx.wdtype), None


def short_conv_silu(x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """Causal depthwise conv (kernel [C, 1, W]) over time then SiLU; x: [B, T, C]."""
    if _eltwise_kernels(x) and weight.shape[-1] <= 8:
        return _ShortConv.apply(x, weight)
    W = weight.shape[-1]
    xt = F.pad(x.transpose(1, 2), (W - 1, 0))
    y = F.conv1d(xt, weight.to(x.dtype), groups=x.shape[-1])
    return F.silu(y).transpose(1, 2)


def gated_rms_norm(x: torch.Tensor, gate: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """RMSNorm over the last dim, times weight, times sigmoid(gate)."""
    if _eltwise_kernels(x) and type(weight).__name__ != "DTensor":
        return _GatedNorm.apply(x, gate, weight, eps)
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * weight.float()
    return (y * torch.sigmoid(gate.float())).to(x.dtype)
