"""The decayed-Gram KDA kernels against the column-loop formulation (fp32).
New kernels, not yet validated on a B200: run with TTB_KDA_KERNEL_TESTS=1."""
import os

import pytest
import torch

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(os.environ.get("TTB_KDA_KERNEL_TESTS") != "1",
                                 reason="KDA Gram kernels not yet validated on a B200; opt in explicitly")]


@pytest.mark.parametrize("strict", [True, False])
@pytest.mark.parametrize("N,C,K", [(5, 64, 128), (40, 64, 64)])
def test_kda_gram_kernels_match_loop(strict, N, C, K, monkeypatch):
    from torchtitan_b200.ops import kda

    torch.manual_seed(0)
    a, b = (torch.randn(N, C, K, device="cuda") for _ in range(2))
    G = (-torch.rand(N, C, K, device="cuda") * 0.3).cumsum(1)
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
