"""The decayed-Gram KDA kernels against the column-loop formulation (fp32),
and the inter-chunk recurrence kernels against the batched-matmul loop."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("strict", [True, False])
@pytest.mark.parametrize("N,C,K,rate", [(5, 64, 128, 0.3), (40, 64, 64, 0.3), (7, 32, 128, 0.3),
                                        (5, 64, 128, 5.0)])
def test_kda_gram_kernels_match_loop(strict, N, C, K, rate, monkeypatch):
    """rate 5.0: log decay down to -320 over a chunk (factorised exponentials stay <= 1)."""
    from torchtitan_b200.ops import kda

    torch.manual_seed(0)
    a, b = (torch.randn(N, C, K, device="cuda") for _ in range(2))
    G = (-torch.rand(N, C, K, device="cuda") * rate).cumsum(1)
    dout = torch.randn(N, C, C, device="cuda")
    outs = {}
    for flag in ("0", "1"):
        monkeypatch.setenv("TTB_KDA_KERNEL", flag)
        aa, bb, gg = (t.clone().requires_grad_() for t in (a, b, G))
        y = kda.decayed_gram(aa, bb, gg, strict)
        (y * dout).sum().backward()
        outs[flag] = (y.detach(), aa.grad, bb.grad, gg.grad)
    for x, y in zip(outs["0"], outs["1"]):
        torch.testing.assert_close(y, x, rtol=2e-4, atol=2e-4)


@pytest.mark.parametrize("BH,NT,C,K,V", [(3, 5, 64, 128, 128), (2, 3, 64, 64, 96)])
def test_kda_chunk_scan_kernel_matches_loop(BH, NT, C, K, V):
    """The inter-chunk recurrence kernels (forward and backward) against the batched-matmul loop."""
    from torchtitan_b200.ops import kda

    torch.manual_seed(1)
    u = torch.randn(BH, NT, C, V, device="cuda")
    w, qg, kd = (0.1 * torch.randn(BH, NT, C, K, device="cuda") for _ in range(3))
    A = 0.1 * torch.randn(BH, NT, C, C, device="cuda").tril()
    dec = torch.rand(BH, NT, K, device="cuda") * 0.5 + 0.5
    do = torch.randn(BH, NT, C, V, device="cuda")
    res = []
    for fn in (kda._scan_ref, kda._ChunkScan.apply):
        xs = [t.clone().requires_grad_() for t in (u, w, qg, A, kd, dec)]
        o, S = fn(*xs)
        (o * do).sum().backward()
        res.append([o.detach(), S.detach()] + [x.grad for x in xs])
    for got, want in zip(res[1], res[0]):
        torch.testing.assert_close(got, want, rtol=1e-3, atol=1e-3)


def test_chunk_kda_with_scan_kernel_matches_recurrence(monkeypatch):
    from torchtitan_b200.ops import kda

    torch.manual_seed(2)
    B, T, H, K, V = 1, 200, 2, 64, 64
    q, k = (torch.randn(B, T, H, K, device="cuda") for _ in range(2))
    v = torch.randn(B, T, H, V, device="cuda")
    g = -torch.rand(B, T, H, K, device="cuda") * 0.2
    beta = torch.rand(B, T, H, device="cuda")
    monkeypatch.setenv("TTB_KDA_KERNEL", "1")
    o, _ = kda.chunk_kda(q, k, v, g, beta)
    ref, _ = kda.naive_recurrent_kda(q, k, v, g, beta)
    torch.testing.assert_close(o.float(), ref, rtol=2e-3, atol=2e-3)


def _rel(a, b):
    return float((a.float() - b.float()).norm() / (b.float().norm() + 1e-12))


@pytest.mark.parametrize("BH,NT,with_state", [(3, 5, False), (2, 9, True)])
def test_kda_state_kernels_match_loop(BH, NT, with_state):
    """The tcgen05 state-passing recurrence (bf16 operands, fp32 state) against the fp32
    batched-matmul loop: outputs, final state, and the gradients of every input including the
    initial state, with a gradient on the final state too."""
    from torchtitan_b200.ops import kda

    torch.manual_seed(3)
    C, K, V = 64, 128, 128
    u = torch.randn(BH, NT, C, V, device="cuda")
    w, qg, kd = (0.05 * torch.randn(BH, NT, C, K, device="cuda") for _ in range(3))
    A = 0.1 * torch.randn(BH, NT, C, C, device="cuda").tril()
    dec = torch.rand(BH, NT, K, device="cuda") * 0.5 + 0.5
    S0 = torch.randn(BH, K, V, device="cuda") if with_state else None
    do = torch.randn(BH, NT, C, V, device="cuda")
    dfin = torch.randn(BH, K, V, device="cuda")
    res = []
    for fn in (lambda *x: kda._scan_ref(*x), lambda *x: kda._StateScan.apply(*x)):
        xs = [t.clone().requires_grad_() for t in (u, w, qg, A, kd, dec)]
        s0 = S0.clone().requires_grad_() if with_state else None
        o, S = fn(*xs, s0)
        ((o * do).sum() + (S * dfin).sum()).backward()
        res.append([o.detach(), S.detach()] + [x.grad for x in xs] + ([s0.grad] if with_state else []))
    from torchtitan_b200.ops._ext import ext

    assert ext().kda_state_error_code(True) == 0
    names = ["o", "S", "du", "dw", "dqg", "dA", "dkd", "ddec", "dS0"]
    for n, got, want in zip(names, res[1], res[0]):
        assert _rel(got, want) < 3e-2, (n, _rel(got, want))


def test_chunk_kda_state_kernel_matches_recurrence():
    """Whole chunked KDA at K = V = 128 (the tcgen05 state path) against the token recurrence,
    with a sequence that is not a multiple of the chunk."""
    from torchtitan_b200.ops import kda

    torch.manual_seed(2)
    B, T, H, K, V = 1, 300, 2, 128, 128
    q, k = (torch.randn(B, T, H, K, device="cuda") for _ in range(2))
    v = torch.randn(B, T, H, V, device="cuda")
    g = -torch.rand(B, T, H, K, device="cuda") * 0.2
    beta = torch.rand(B, T, H, device="cuda")
    o, S = kda.chunk_kda(q, k, v, g, beta, output_final_state=True)
    ref, Sref = kda.naive_recurrent_kda(q, k, v, g, beta)
    assert _rel(o, ref) < 2e-2 and _rel(S, Sref) < 2e-2


@pytest.mark.parametrize("T", [200, 256])
def test_chunk_kda_prep_kernel_matches_torch_ops(T, monkeypatch):
    """The one-pass chunk preparation (csrc/kda_prep.cu) against the PyTorch ops it replaces:
    outputs, final state and the gradients of q, k, v, g, beta (T = 200 pads the last chunk)."""
    from torchtitan_b200.ops import kda

    torch.manual_seed(5)
    B, H, K, V = 2, 3, 64, 64
    base = [torch.randn(B, T, H, K, device="cuda"), torch.randn(B, T, H, K, device="cuda"),
            torch.randn(B, T, H, V, device="cuda"), -torch.rand(B, T, H, K, device="cuda") * 0.3,
            torch.rand(B, T, H, device="cuda")]
    s0 = torch.randn(B, H, K, V, device="cuda") * 0.1
    do = torch.randn(B, T, H, V, device="cuda")
    dS = torch.randn(B, H, K, V, device="cuda")
    res = {}
    for flag in ("0", "1"):
        monkeypatch.setenv("TTB_KDA_PREP", flag)
        xs = [t.clone().requires_grad_() for t in base]
        o, S = kda.chunk_kda(*xs, initial_state=s0, output_final_state=True)
        ((o.float() * do).sum() + (S * dS).sum()).backward()
        res[flag] = [o.detach().float(), S.detach()] + [x.grad for x in xs]
    for name, a, b in zip(["o", "S", "dq", "dk", "dv", "dg", "dbeta"], res["1"], res["0"]):
        assert _rel(a, b) < 1e-4, (name, _rel(a, b))
