"""The fused routing-selection kernel (``csrc/router_topk.cu``) against the PyTorch router:
same experts chosen (as sets per token) and the same per-expert counts.  The kernel is the
default on CUDA (TTB_ROUTER_KERNEL=0 selects PyTorch)."""
import os

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("E,k,score,groups", [(8, 2, "softmax", None), (64, 8, "sigmoid", None),
                                              (256, 8, "sigmoid", (8, 4)), (128, 8, "softmax", None)])
def test_router_kernel_matches_torch(E, k, score, groups, monkeypatch):
    from torchtitan_b200.models.common.moe import TokenChoiceTopKRouter

    torch.manual_seed(0)
    r = TokenChoiceTopKRouter(64, E, k, score_func=score, route_norm=True,
                              num_expert_groups=groups[0] if groups else None,
                              num_limited_groups=groups[1] if groups else None).cuda()
    r.init_weights(0.5)
    x = torch.randn(1000, 64, device="cuda", dtype=torch.bfloat16)
    bias = 0.01 * torch.randn(E, device="cuda")
    r.gate.weight.data = r.gate.weight.data.bfloat16()
    outs = {}
    for flag in ("0", "1"):
        monkeypatch.setenv("TTB_ROUTER_KERNEL", flag)
        outs[flag] = r(x, bias)
    (t0, i0, c0, _), (t1, i1, c1, _) = outs["0"], outs["1"]
    assert torch.equal(i0.sort(-1).values, i1.sort(-1).values)
    assert torch.equal(c0, c1)
    torch.testing.assert_close(t0.gather(1, i0.argsort(-1)), t1.gather(1, i1.argsort(-1)))
