"""KDA short causal conv + SiLU and gated RMSNorm kernels (``csrc/kda_eltwise.cu``) against
the PyTorch formulations, forward and backward.  The kernels are the default
on CUDA (TTB_KDA_ELTWISE=0 selects PyTorch)."""
import os

import pytest
import torch

pytestmark = pytest.mark.gpu


def _both(fn, args, monkeypatch, grads_of):
    res = {}
    for flag in ("0", "1"):
        monkeypatch.setenv("TTB_KDA_ELTWISE", flag)
        xs = [a.clone().requires_grad_() if i in grads_of else a for i, a in enumerate(args)]
        y = fn(*xs)
        torch.manual_seed(5)
        y.backward(torch.randn(y.shape, device=y.device, dtype=y.dtype))  # same values whatever y's strides
        res[flag] = [y.float()] + [xs[i].grad.float() for i in grads_of]
    return res


@pytest.mark.parametrize("B,T,C,W", [(2, 300, 512, 4), (1, 77, 96, 3)])
def test_short_conv_kernel(B, T, C, W, monkeypatch):
    from torchtitan_b200.ops import kda

    torch.manual_seed(0)
    x = torch.randn(B, T, C, device="cuda", dtype=torch.bfloat16)
    w = 0.3 * torch.randn(C, 1, W, device="cuda")
    res = _both(kda.short_conv_silu, (x, w), monkeypatch, (0, 1))
    for a, b in zip(res["1"], res["0"]):
        torch.testing.assert_close(a, b, rtol=2e-2, atol=2e-2 * float(b.abs().max()))


@pytest.mark.parametrize("R,D", [(600, 128), (33, 2304)])
def test_gated_norm_kernel(R, D, monkeypatch):
    from torchtitan_b200.ops import kda

    torch.manual_seed(1)
    x = torch.randn(R, D, device="cuda", dtype=torch.bfloat16)
    z = torch.randn(R, D, device="cuda", dtype=torch.bfloat16)
    g = 1 + 0.1 * torch.randn(D, device="cuda")
    res = _both(lambda a, b, c: kda.gated_rms_norm(a, b, c, 1e-6), (x, z, g), monkeypatch, (0, 1, 2))
    for a, b in zip(res["1"], res["0"]):
        torch.testing.assert_close(a, b, rtol=2e-2, atol=2e-2 * float(b.abs().max()))


def test_kda_gate_kernel(monkeypatch):
    from torchtitan_b200.ops import kda

    torch.manual_seed(2)
    x = torch.randn(2, 300, 4, 64, device="cuda", dtype=torch.bfloat16)
    A = torch.randn(4, device="cuda")
    b = 0.1 * torch.randn(4 * 64, device="cuda")
    res = _both(kda.kda_gate, (x, A, b), monkeypatch, (0, 1, 2))
    for a, c in zip(res["1"], res["0"]):
        torch.testing.assert_close(a, c, rtol=2e-2, atol=2e-2 * float(c.abs().max()))
