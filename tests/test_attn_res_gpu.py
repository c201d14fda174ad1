"""The fused block attention-residual kernel (``csrc/attn_res.cu``) against the PyTorch
formulation, forward and backward (inputs, pseudo-query and norm weight).  The kernel is the
default on CUDA (TTB_ATTNRES_KERNEL=0 selects PyTorch)."""
import os

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("nb,D", [(1, 256), (5, 2304), (9, 4096)])
def test_attn_res_kernel_matches_torch(nb, D, monkeypatch):
    from torchtitan_b200.models.common.attn_res import block_attn_res
    from torchtitan_b200.models.common.layers import Linear, RMSNorm

    torch.manual_seed(0)
    q = Linear(D, 1).cuda()
    q.weight.data.normal_(0, 0.05)
    norm = RMSNorm(D, 1e-6).cuda()
    norm.weight.data = 1 + 0.1 * torch.randn(D, device="cuda")
    vs = [torch.randn(2, 300, D, device="cuda", dtype=torch.bfloat16) for _ in range(nb)]
    dout = torch.randn(2, 300, D, device="cuda", dtype=torch.bfloat16)
    res = {}
    for flag in ("0", "1"):
        monkeypatch.setenv("TTB_ATTNRES_KERNEL", flag)
        xs = [v.clone().requires_grad_() for v in vs]
        for p in (q.weight, norm.weight):
            p.grad = None
        o = block_attn_res(xs[:-1], xs[-1], q.weight, norm)
        o.backward(dout)
        res[flag] = [o.float()] + [x.grad.float() for x in xs] + [q.weight.grad.clone(), norm.weight.grad.clone()]
    for a, b in zip(res["1"], res["0"]):
        torch.testing.assert_close(a, b, rtol=3e-2, atol=3e-2 * float(b.abs().max()))
