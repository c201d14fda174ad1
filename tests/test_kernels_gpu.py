"""Numerics of the sm_100a kernels against plain-PyTorch fp32 restatements."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ext():
    from torchtitan_b200.ops._ext import ext as _e

    return _e()


def _rel(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 1024), (1000, 776, 520), (37, 24, 8), (4096, 4096, 4096)])
@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, False), (True, True)])
def test_gemm(ext, M, N, K, a_mn, b_mn):
    if (a_mn and M % 8) or (b_mn and N % 8):
        pytest.skip("TMA needs the contiguous dimension to be a multiple of 8")
    torch.manual_seed(0)
    A = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    B = torch.randn(N, K, device="cuda", dtype=torch.bfloat16)
    a_in = A.t().contiguous() if a_mn else A
    b_in = B.t().contiguous() if b_mn else B
    D = ext.gemm(a_in, b_in, a_mn, b_mn)
    ref = A.float() @ B.float().t()
    torch.cuda.synchronize()
    assert ext.gemm_error_code(True) == 0
    assert D.shape == (M, N)
    assert _rel(D, ref) < 1e-2


def test_linear_autograd():
    from torchtitan_b200 import ops

    torch.manual_seed(1)
    x = torch.randn(4, 96, 256, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = torch.randn(384, 256, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    y = ops.linear(x, w)
    g = torch.randn_like(y)
    y.backward(g)
    xr, wr = x.detach().float().requires_grad_(), w.detach().float().requires_grad_()
    yr = xr @ wr.t()
    yr.backward(g.float())
    assert _rel(y, yr) < 1e-2
    assert _rel(x.grad, xr.grad) < 1e-2
    assert _rel(w.grad, wr.grad) < 1e-2


@pytest.mark.parametrize("rows,dim", [(300, 256), (300, 4096), (300, 2304), (5000, 4096), (3001, 8192),
                                      (1500, 16384), (7001, 1024)])
def test_rmsnorm(rows, dim):
    """Includes row counts above the persistent grid (several rows per CTA, odd tails)."""
    from torchtitan_b200 import ops

    torch.manual_seed(2)
    x = torch.randn(rows, dim, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = (1 + 0.1 * torch.randn(dim, device="cuda")).to(torch.bfloat16).requires_grad_()
    y = ops.rms_norm(x, w, 1e-5)
    g = torch.randn_like(y)
    y.backward(g)
    xr, wr = x.detach().float().requires_grad_(), w.detach().float().requires_grad_()
    yr = xr * torch.rsqrt(xr.pow(2).mean(-1, keepdim=True) + 1e-5) * wr
    yr.backward(g.float())
    assert _rel(y, yr) < 1e-2
    assert _rel(x.grad, xr.grad) < 2e-2
    assert _rel(w.grad, wr.grad) < 2e-2


def test_rope():
    from torchtitan_b200 import ops
    from torchtitan_b200.models.common.rope import precompute_rope
    from torchtitan_b200.ops import reference as R

    torch.manual_seed(3)
    cos, sin = precompute_rope(128, 512, 500000.0, "llama")
    cos, sin = cos.cuda(), sin.cuda()
    x = torch.randn(2, 512, 8, 128, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    y = ops.rope(x, cos, sin)
    g = torch.randn_like(y)
    y.backward(g)
    xr = x.detach().float().requires_grad_()
    yr = R.rope(xr, cos, sin)
    yr.backward(g.float())
    assert _rel(y, yr) < 1e-2
    assert _rel(x.grad, xr.grad) < 1e-2


def test_swiglu():
    from torchtitan_b200 import ops

    torch.manual_seed(4)
    a = torch.randn(64, 1024, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    b = torch.randn(64, 1024, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    y = ops.swiglu(a, b)
    g = torch.randn_like(y)
    y.backward(g)
    ar, br = a.detach().float().requires_grad_(), b.detach().float().requires_grad_()
    yr = torch.nn.functional.silu(ar) * br
    yr.backward(g.float())
    assert _rel(y, yr) < 1e-2
    assert _rel(a.grad, ar.grad) < 2e-2
    assert _rel(b.grad, br.grad) < 2e-2


@pytest.mark.parametrize("V", [2048, 128256])
def test_cross_entropy(V):
    from torchtitan_b200 import ops

    torch.manual_seed(5)
    T = 257
    logits = (3 * torch.randn(T, V, device="cuda")).to(torch.bfloat16).requires_grad_()
    labels = torch.randint(0, V, (T,), device="cuda")
    labels[::7] = -100
    loss = ops.cross_entropy_sum(logits, labels)
    loss.backward(torch.tensor(0.5, device="cuda"))
    lr_ = logits.detach().float().requires_grad_()
    ref = torch.nn.functional.cross_entropy(lr_, labels, reduction="sum", ignore_index=-100)
    ref.backward(torch.tensor(0.5, device="cuda"))
    assert abs(loss.item() - ref.item()) / abs(ref.item()) < 1e-3
    assert _rel(logits.grad, lr_.grad) < 2e-2


@pytest.mark.parametrize("pdtype", [torch.float32, torch.bfloat16])
def test_adamw(pdtype):
    from torchtitan_b200 import ops
    from torchtitan_b200.ops import reference as R

    torch.manual_seed(6)
    shapes = [(1000,), (300, 257), (70000,)]
    ps = [torch.randn(s, device="cuda").to(pdtype) for s in shapes]
    gs = [torch.randn(s, device="cuda") for s in shapes]
    ms = [torch.randn(s, device="cuda").abs() * 0.1 for s in shapes]
    vs = [torch.randn(s, device="cuda").abs() * 0.1 for s in shapes]
    rp = [p.float().clone() for p in ps]
    rm = [m.clone() for m in ms]
    rv = [v.clone() for v in vs]
    kw = dict(lr=1e-3, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1, step=3)
    ops.fused_adamw_(ps, gs, ms, vs, **kw)
    R.adamw_(rp, gs, rm, rv, **kw)
    tol = 1e-5 if pdtype == torch.float32 else 1e-2
    for p, r in zip(ps, rp):
        assert _rel(p, r) < tol
    for m, r in zip(ms, rm):
        assert _rel(m, r) < 1e-5


def _attn_ref(q, k, v, causal, scale):
    from torchtitan_b200.ops import reference as R

    return R.attention(q.float(), k.float(), v.float(), causal, scale)


@pytest.mark.parametrize(
    "B,Sq,Sk,H,Hk,D,Dv,causal",
    [
        (1, 128, 128, 2, 2, 128, 128, True),
        (2, 256, 256, 4, 2, 128, 128, True),
        (1, 384, 384, 4, 1, 128, 128, False),
        (1, 200, 200, 2, 2, 128, 128, True),
        (1, 128, 384, 2, 2, 128, 128, True),
        (1, 256, 256, 2, 2, 64, 64, True),
        (1, 256, 256, 4, 4, 192, 128, True),
    ],
)
def test_attention(ext, B, Sq, Sk, H, Hk, D, Dv, causal):
    from torchtitan_b200 import ops

    torch.manual_seed(7)
    q = torch.randn(B, Sq, H, D, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    k = torch.randn(B, Sk, Hk, D, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    v = torch.randn(B, Sk, Hk, Dv, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    scale = 1.0 / math.sqrt(D)
    o = ops.attention(q, k, v, causal=causal, scale=scale)
    g = torch.randn_like(o)
    o.backward(g)
    qr, kr, vr = (t.detach().float().requires_grad_() for t in (q, k, v))
    orf = _attn_ref(qr, kr, vr, causal, scale)
    orf.backward(g.float())
    torch.cuda.synchronize()
    assert ext.attn_error_code(True) == 0
    assert _rel(o, orf) < 2e-2
    assert _rel(q.grad, qr.grad) < 3e-2
    assert _rel(k.grad, kr.grad) < 3e-2
    assert _rel(v.grad, vr.grad) < 3e-2


def test_grad_clip_kernels(ext):
    torch.manual_seed(8)
    xs = [torch.randn(s, device="cuda") for s in [(1000,), (333, 77), (70001,)]] + \
         [torch.randn(4096, device="cuda").bfloat16()]
    ref = sum(float(x.float().pow(2).sum()) for x in xs)
    tot = ext.multi_sumsq(xs)
    assert abs(tot.item() - ref) / ref < 1e-5
    before = [x.float().clone() for x in xs]
    ext.multi_clip_scale(xs, tot, 1.0)
    coef = 1.0 / (ref ** 0.5 + 1e-6)
    for x, b in zip(xs, before):
        assert _rel(x, b * coef) < 1e-2


@pytest.mark.parametrize("E,D,H", [(8, 256, 512), (4, 2304, 1024)])
def test_grouped_swiglu_experts(E, D, H):
    from torchtitan_b200.ops.moe import _reference, grouped_swiglu

    torch.manual_seed(9)
    counts = torch.tensor([0, 300, 5, 128][:E] + [77] * max(0, E - 4), device="cuda")
    n = int(counts.sum())
    x = (torch.randn(n, D, device="cuda") * 0.5).bfloat16().requires_grad_()
    w = [(torch.randn(E, H, D, device="cuda") * 0.05).bfloat16().requires_grad_(),
         (torch.randn(E, D, H, device="cuda") * 0.05).bfloat16().requires_grad_(),
         (torch.randn(E, H, D, device="cuda") * 0.05).bfloat16().requires_grad_()]
    y = grouped_swiglu(x, w[0], w[1], w[2], counts)
    g = torch.randn_like(y)
    y.backward(g)
    xr = x.detach().float().requires_grad_()
    wr = [t.detach().float().requires_grad_() for t in w]
    yr = _reference(xr, wr[0], wr[1], wr[2], counts)
    yr.backward(g.float())
    assert _rel(y, yr) < 2e-2
    assert _rel(x.grad, xr.grad) < 3e-2
    for a, b in zip(w, wr):
        assert _rel(a.grad, b.grad) < 3e-2


def test_attention_padded_head_dims():
    from torchtitan_b200 import ops

    torch.manual_seed(10)
    q = torch.randn(1, 128, 2, 111, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    k = torch.randn(1, 128, 2, 111, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    v = torch.randn(1, 128, 2, 74, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    o = ops.attention(q, k, v, causal=True)
    o.sum().backward()
    ref = _attn_ref(q.detach(), k.detach(), v.detach(), True, 111 ** -0.5)
    assert o.shape == (1, 128, 2, 74) and _rel(o, ref) < 2e-2 and q.grad.shape == q.shape


def test_linear_unaligned_dims():
    from torchtitan_b200 import ops

    x = torch.randn(64, 250, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = torch.randn(3, 250, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    y = ops.linear(x, w)
    y.sum().backward()
    assert y.shape == (64, 3) and _rel(y, x.float() @ w.float().t()) < 1e-2
    assert w.grad.shape == w.shape and x.grad.shape == x.shape


def test_adamw_master_with_bf16_copy():
    from torchtitan_b200 import ops
    from torchtitan_b200.ops import reference as R

    torch.manual_seed(12)
    p = torch.randn(4096 + 4, device="cuda")
    g = torch.randn_like(p).bfloat16()
    m, v = torch.zeros_like(p), torch.zeros_like(p)
    copy = torch.empty_like(p, dtype=torch.bfloat16)
    rp, rm, rv = p.clone(), m.clone(), v.clone()
    kw = dict(lr=1e-3, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1, step=1)
    ops.fused_adamw_([p], [g], [m], [v], copies=[copy], **kw)
    R.adamw_([rp], [g.float()], [rm], [rv], **kw)
    assert _rel(p, rp) < 1e-5 and _rel(copy, rp) < 1e-2


@pytest.mark.parametrize("M,N,K", [(256, 256, 64), (512, 768, 1024), (1000, 776, 520), (4096, 4096, 4096)])
@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, False), (True, True)])
def test_gemm_2sm(ext, M, N, K, a_mn, b_mn):
    torch.manual_seed(13)
    A = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    B = torch.randn(N, K, device="cuda", dtype=torch.bfloat16)
    D = ext.gemm_2sm(A.t().contiguous() if a_mn else A, B.t().contiguous() if b_mn else B, a_mn, b_mn)
    torch.cuda.synchronize()
    assert ext.gemm2_error_code(True) == 0
    assert _rel(D, A.float() @ B.float().t()) < 1e-2


def test_adamw_fused_clip(ext):
    from torchtitan_b200 import ops
    from torchtitan_b200.ops import reference as R

    torch.manual_seed(14)
    p = torch.randn(10000, device="cuda")
    g = torch.randn_like(p) * 3
    m, v = torch.zeros_like(p), torch.zeros_like(p)
    rp, rm, rv = p.clone(), m.clone(), v.clone()
    total = g.pow(2).sum()
    coef = min(1.0, 1.0 / (total.sqrt().item() + 1e-6))
    kw = dict(lr=1e-3, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1, step=2)
    ops.fused_adamw_([p], [g], [m], [v], clip_total=total, clip_max=1.0, **kw)
    R.adamw_([rp], [g * coef], [rm], [rv], **kw)
    assert _rel(p, rp) < 1e-5 and _rel(m, rm) < 1e-5


def test_grouped_swiglu_padded_matches_unpadded():
    from torchtitan_b200 import ops
    from torchtitan_b200.ops.grouped import expert_segments, grouped_swiglu_padded

    torch.manual_seed(0)
    E, D, H = 3, 256, 384
    counts = torch.tensor([70, 0, 200], device="cuda")
    x = torch.randn(int(counts.sum()), D, device="cuda", dtype=torch.bfloat16)
    w1, w3 = (torch.randn(E, H, D, device="cuda", dtype=torch.bfloat16) * 0.05 for _ in range(2))
    w2 = torch.randn(E, D, H, device="cuda", dtype=torch.bfloat16) * 0.05
    tg, kst, kln, P = expert_segments(counts)
    xp = torch.zeros(P, D, device="cuda", dtype=torch.bfloat16)
    xp[0:70] = x[:70]
    xp[int(kst[2]):int(kst[2]) + 200] = x[70:]
    y = ops.grouped_swiglu(x, w1, w2, w3, counts)
    yp = grouped_swiglu_padded(xp, w1, w2, w3, counts)
    torch.testing.assert_close(yp[:70], y[:70], rtol=0, atol=0)
    torch.testing.assert_close(yp[int(kst[2]):int(kst[2]) + 200], y[70:], rtol=0, atol=0)


@pytest.mark.parametrize("D", [64, 128])
def test_attention_lse_output_and_gradient(D):
    """The flash kernel's log-sum-exp output and the dlse term of its backward (used for
    attention sinks) against fp32 PyTorch."""
    from torchtitan_b200.ops.attention import _attention_lse_ref, attention_with_lse

    torch.manual_seed(0)
    B, S, H, Hk = 1, 256, 8, 2
    q, k, v = (torch.randn(B, S, h, D, device="cuda", dtype=torch.bfloat16) for h in (H, Hk, Hk))
    go = torch.randn(B, S, H, D, device="cuda")
    gl = torch.randn(B, S, H, device="cuda")
    outs = []
    for fn in (attention_with_lse, _attention_lse_ref):
        qq, kk, vv = (t.detach().float().requires_grad_() if fn is _attention_lse_ref else
                      t.detach().clone().requires_grad_() for t in (q, k, v))
        o, lse = fn(qq, kk, vv, True, D ** -0.5)
        ((o.float() * go).sum() + (lse.float() * gl).sum()).backward()
        outs.append((o.float(), lse.float(), qq.grad.float(), kk.grad.float(), vv.grad.float()))
    for a, b in zip(*outs):
        torch.testing.assert_close(a, b, rtol=3e-2, atol=3e-2)


@pytest.mark.parametrize("S,lens,D", [(320, [[1, 37, 130, 152], [320]], 128),
                                     (1000, [[300, 1, 255, 444], [129, 128, 743]], 64),
                                     (777, [[500, 277], [1, 1, 775]], 96)])
def test_document_attention(ext, S, lens, D):
    """Packed documents: the block-causal mask applied inside the flash kernels (one launch,
    per-token document start/end tables) against fp32 PyTorch with the dense mask, forward and
    backward, for documents that start and end inside tiles."""
    from torchtitan_b200 import ops
    from torchtitan_b200.models.common.attention import document_causal_mask

    torch.manual_seed(9)
    B, H, Hk = 2, 4, 2
    doc = torch.tensor([sum(([i] * n for i, n in enumerate(r)), []) for r in lens], device="cuda")
    q = torch.randn(B, S, H, D, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    k = torch.randn(B, S, Hk, D, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    v = torch.randn(B, S, Hk, D, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    o = ops.document_attention(q, k, v, doc)
    g = torch.randn_like(o)
    o.backward(g)
    qr, kr, vr = (t.detach().float().requires_grad_() for t in (q, k, v))
    orf = torch.nn.functional.scaled_dot_product_attention(
        qr.transpose(1, 2), kr.repeat_interleave(2, 2).transpose(1, 2), vr.repeat_interleave(2, 2).transpose(1, 2),
        attn_mask=document_causal_mask(doc)).transpose(1, 2)
    orf.backward(g.float())
    torch.cuda.synchronize()
    assert ext.attn_error_code(True) == 0
    assert _rel(o, orf) < 2e-2
    for a, b in ((q.grad, qr.grad), (k.grad, kr.grad), (v.grad, vr.grad)):
        assert _rel(a, b) < 3e-2


def test_grouped_bmm_and_batched_newton_schulz(ext):
    """Equal-shape stacks through one grouped GEMM (the batched path of ops.matmul used by
    Muon's Newton-Schulz on expert stacks) against fp32 torch.bmm, and the batched iteration
    against the per-matrix one."""
    from torchtitan_b200.components.optimizer import zeropower_via_newtonschulz5
    from torchtitan_b200.ops.gemm import bmm_grouped

    torch.manual_seed(4)
    a = torch.randn(6, 256, 192, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(6, 192, 320, device="cuda", dtype=torch.bfloat16)
    want = torch.bmm(a.float(), b.float())
    assert _rel(bmm_grouped(a, b), want) < 1e-2
    x = torch.randn(8, 128, 384, device="cuda")
    with torch.no_grad():
        batched = zeropower_via_newtonschulz5(x)
        single = torch.stack([zeropower_via_newtonschulz5(m) for m in x])
    assert _rel(batched, single) < 2e-2


def test_adamw_and_sumsq_device_table_path(ext):
    """Updates with more chunks than one kernel-argument table holds go through the device-memory
    chunk table and one persistent launch: two steps on the same tensors (table reused), then a
    different tensor set (table rebuilt), against fp32 PyTorch; same for the sum of squares."""
    from torchtitan_b200 import ops
    from torchtitan_b200.ops import reference as R

    torch.manual_seed(12)
    kw = dict(lr=1e-3, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1)
    for n_t in (700, 650):
        shapes = [(1000 + 8 * (i % 5),) for i in range(n_t)] + [(70000 * 3,)]
        ps = [torch.randn(s, device="cuda") for s in shapes]
        gs = [torch.randn(s, device="cuda").bfloat16() for s in shapes]
        ms = [torch.zeros(s, device="cuda") for s in shapes]
        vs = [torch.zeros(s, device="cuda") for s in shapes]
        rp, rm, rv = [p.clone() for p in ps], [m.clone() for m in ms], [v.clone() for v in vs]
        for step in (1, 2):
            ops.fused_adamw_(ps, gs, ms, vs, step=step, **kw)
            R.adamw_(rp, [g.float() for g in gs], rm, rv, step=step, **kw)
        for p, r in zip(ps[::50], rp[::50]):
            assert _rel(p, r) < 1e-5
        tot = ext.multi_sumsq(gs)
        ref = sum(float(g.float().pow(2).sum()) for g in gs)
        assert abs(tot.item() - ref) / ref < 1e-5
