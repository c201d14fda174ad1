"""KDA chunked formulation vs the token recurrence (CPU, fp64)."""
import torch

from torchtitan_b200.ops import kda


def _inputs(B=1, T=40, H=2, K=8, V=8, seed=0, dtype=torch.float64):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, T, H, K, generator=g, dtype=dtype)
    k = torch.randn(B, T, H, K, generator=g, dtype=dtype)
    v = torch.randn(B, T, H, V, generator=g, dtype=dtype)
    graw = torch.randn(B, T, H, K, generator=g, dtype=dtype)
    A_log = torch.log(torch.empty(H, dtype=dtype).uniform_(1, 16, generator=g))
    gate = kda.kda_gate(graw, A_log, None).to(dtype)
    beta = torch.sigmoid(torch.randn(B, T, H, generator=g, dtype=dtype))
    return q, k, v, gate, beta


def test_chunk_matches_recurrence():
    q, k, v, g, beta = _inputs()
    o_ref, S_ref = kda.naive_recurrent_kda(q, k, v, g, beta)
    o, S = kda.chunk_kda(q, k, v, g, beta, chunk_size=16, output_final_state=True)
    assert torch.allclose(o.double(), o_ref.double(), atol=1e-4, rtol=1e-4)
    assert torch.allclose(S.double(), S_ref.double(), atol=1e-4, rtol=1e-4)


def test_chunk_grads_match_recurrence():
    q, k, v, g, beta = _inputs(T=24, seed=1)
    ins = [t.clone().requires_grad_() for t in (q, k, v, g, beta)]
    ins2 = [t.clone().requires_grad_() for t in (q, k, v, g, beta)]
    o, _ = kda.chunk_kda(*ins, chunk_size=8)
    o_ref, _ = kda.naive_recurrent_kda(*ins2)
    w = torch.randn_like(o_ref)
    (o * w).sum().backward()
    (o_ref * w).sum().backward()
    for a, b in zip(ins, ins2):
        assert torch.allclose(a.grad.double(), b.grad.double(), atol=1e-4, rtol=1e-3)


def test_decayed_gram_gradcheck():
    g = torch.Generator().manual_seed(3)
    a = torch.randn(2, 5, 3, generator=g, dtype=torch.float64, requires_grad=True)
    b = torch.randn(2, 5, 3, generator=g, dtype=torch.float64, requires_grad=True)
    G = (-torch.rand(2, 5, 3, generator=g, dtype=torch.float64)).cumsum(1).requires_grad_()
    for strict in (True, False):
        assert torch.autograd.gradcheck(lambda a, b, G: kda.decayed_gram(a, b, G, strict), (a, b, G))


def test_decayed_gram_backward_closed_form():
    """The kernel's backward uses dG = a * da - b * db; check it against autograd of the loop."""
    from torchtitan_b200.ops.kda import decayed_gram

    torch.manual_seed(0)
    N, C, K = 3, 16, 8
    a, b = torch.randn(N, C, K, dtype=torch.float64), torch.randn(N, C, K, dtype=torch.float64)
    G = (-torch.rand(N, C, K, dtype=torch.float64)).cumsum(1)
    for strict in (True, False):
        dout = torch.randn(N, C, C, dtype=torch.float64)
        aa, bb, gg = (t.clone().requires_grad_() for t in (a, b, G))
        (decayed_gram(aa, bb, gg, strict) * dout).sum().backward()
        i = torch.arange(C)
        mask = (i[:, None] > i[None, :]) if strict else (i[:, None] >= i[None, :])
        w = dout * mask
        e = torch.exp((G[:, :, None, :] - G[:, None, :, :]).clamp(max=0))  # [N, i, j, K]
        da = torch.einsum("nij,nijd,njd->nid", w, e, b)
        db = torch.einsum("nij,nijd,nid->njd", w, e, a)
        torch.testing.assert_close(aa.grad, da)
        torch.testing.assert_close(bb.grad, db)
        torch.testing.assert_close(gg.grad, a * da - b * db)
