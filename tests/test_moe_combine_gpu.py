"""Deterministic MoE dispatch / combine kernels (``csrc/moe_combine.cu``) on a B200: against an
fp32 PyTorch reference (values and every gradient), bitwise repeatable, and the MoE debug
models with the kernels against the PyTorch index ops."""
import importlib

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("weighted,with_base", [(True, True), (False, False)])
def test_dispatch_combine_match_reference(weighted, with_base):
    from torchtitan_b200 import ops

    torch.manual_seed(0)
    T, k, D, E = 1000, 4, 264, 16
    idx = torch.rand(T, E, device="cuda").topk(k, -1).indices
    order = torch.argsort(idx.flatten(), stable=True)
    token_of = order // k
    pos = ops.slot_positions(order, k)
    x = torch.randn(T, D, device="cuda").bfloat16().requires_grad_()
    base = torch.randn(T, D, device="cuda").bfloat16().requires_grad_() if with_base else None
    w = torch.rand(T, k, device="cuda").requires_grad_() if weighted else None
    y = (ops.moe_dispatch(x, token_of, pos).float() * 1.5).bfloat16()  # stands in for the experts
    out = ops.moe_combine(base, y, w, pos, token_of, order)
    g = torch.randn_like(out)
    out.backward(g)
    xr = x.detach().float().requires_grad_()
    br = base.detach().float().requires_grad_() if with_base else None
    wr = w.detach().clone().requires_grad_() if weighted else None
    yr = xr[token_of] * 1.5
    slot_w = wr.flatten()[order][:, None] if weighted else 1.0
    ref = (br if with_base else torch.zeros(T, D, device="cuda")).index_add(0, token_of, yr * slot_w)
    ref.backward(g.float())
    torch.testing.assert_close(out.float(), ref, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(x.grad.float(), xr.grad, rtol=2e-2, atol=2e-2)
    if with_base:
        torch.testing.assert_close(base.grad.float(), br.grad, rtol=1e-2, atol=1e-2)
    if weighted:
        # dot products over D of bf16 rows against the unrounded fp32 reference: compare norms
        assert (w.grad - wr.grad).norm() <= 1e-2 * wr.grad.norm()
    gx = x.grad.clone()  # fixed summation order: a second backward is bitwise the same
    x.grad = None
    ops.moe_combine(base, (ops.moe_dispatch(x, token_of, pos).float() * 1.5).bfloat16(), w, pos, token_of,
                    order).backward(g)
    assert torch.equal(x.grad, gx)


@pytest.mark.parametrize("family,flavor", [("qwen3", "debugmodel_moe"), ("deepseek_v3", "debugmodel")])
def test_moe_models_with_combine_kernels(family, flavor, monkeypatch):
    spec = importlib.import_module(f"torchtitan_b200.models.{family}").model_registry(flavor)
    torch.manual_seed(0)
    with torch.device("cuda"):
        m = spec.model.build()
    m.init_weights(buffer_device=torch.device("cuda"))
    for p in m.parameters():
        p.data = p.data.to(torch.bfloat16)
    tok = torch.randint(0, spec.model.vocab_size, (2, 256), device="cuda")
    res = []
    for flag in ("1", "0"):
        monkeypatch.setenv("TTB_MOE_COMBINE_KERNEL", flag)
        m.zero_grad(set_to_none=True)
        logits = m(tok)
        logits.float().square().mean().backward()
        res.append((logits.float(), [p.grad.float().clone() for p in m.parameters()]))
    torch.testing.assert_close(res[0][0], res[1][0], rtol=2e-2, atol=2e-2)
    # the kernels sum each token's slots in fp32, the index ops round every slot to bf16 and add
    # in bf16: gradients agree to bf16 noise (relative to the model's largest gradient for the
    # tiny ones, e.g. the router's)
    scale = max(float(b.norm()) for b in res[1][1])
    for a, b in zip(res[0][1], res[1][1]):
        assert (a - b).norm() <= 3e-2 * b.norm() + 1e-3 * scale
