"""MXFP8 quantizer and block-scaled tcgen05 GEMM against the CPU definition of
the format (``ops/mx_gemm.py``), and the MXFP8 linear on the kernel against the same
quantized operands on the bf16 GEMM."""
import os

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("R,C", [(128, 128), (130, 200), (1000, 4096)])
def test_mx_quantize_matches_reference(R, C):
    from torchtitan_b200.ops.mx_gemm import mx_quantize, mx_quantize_ref

    torch.manual_seed(0)
    x = (torch.randn(R, C) * torch.logspace(-3, 3, C)).bfloat16()
    codes, sf = mx_quantize(x.cuda())
    rc, rs = mx_quantize_ref(x.float())
    assert torch.equal(codes.cpu(), rc)
    assert torch.equal(sf.cpu(), rs)


@pytest.mark.parametrize("tile_n", [128, 256])
@pytest.mark.parametrize("M,N,K", [(128, 128, 128), (256, 384, 512), (300, 200, 1024), (4096, 4096, 4096),
                                   (640, 1280, 384)])
def test_mx_gemm_matches_dequantized_product(M, N, K, tile_n):
    """Both tile widths; N = 384 and 200 leave the last 256-wide tile with one or no second
    scale record."""
    from torchtitan_b200.ops._ext import ext
    from torchtitan_b200.ops.mx_gemm import mx_dequantize_ref, mx_gemm, mx_quantize

    torch.manual_seed(0)
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.1
    qa, sa = mx_quantize(a)
    qb, sb = mx_quantize(b)
    d = ext().gemm_mxfp8(qa, sa, qb, sb, tile_n)
    torch.cuda.synchronize()
    assert ext().mxgemm_error_code(True) == 0
    ref = (mx_dequantize_ref(qa, sa).cuda() @ mx_dequantize_ref(qb, sb).cuda().t())
    torch.testing.assert_close(d.float(), ref, rtol=2e-2, atol=2e-2 * float(ref.abs().max()) / 50)


def test_mxfp8_linear_kernel_path_matches_fake_quant(monkeypatch):
    """Forward and both backward GEMMs of the MXFP8 linear on the block-scaled kernel against
    the same quantized operands multiplied on the bf16 GEMM."""
    from torchtitan_b200.components.quantization.mx import _MXLinearFn

    torch.manual_seed(3)
    x = torch.randn(256, 512, device="cuda", dtype=torch.bfloat16)
    w = (torch.randn(384, 512, device="cuda") * 0.05).bfloat16()
    dy = torch.randn(256, 384, device="cuda", dtype=torch.bfloat16)
    res = {}
    for flag in ("0", "1"):
        monkeypatch.setenv("TTB_MXFP8_KERNEL", flag)
        xx, ww = x.clone().requires_grad_(), w.clone().requires_grad_()
        y = _MXLinearFn.apply(xx, ww)
        y.backward(dy)
        res[flag] = (y.float(), xx.grad.float(), ww.grad.float())
    for a, b in zip(res["1"], res["0"]):
        torch.testing.assert_close(a, b, rtol=2e-2, atol=2e-2 * float(b.abs().max()) / 20)


@pytest.mark.parametrize("rowwise", [False, True])
def test_f8_quantize_matches_fake_quant(rowwise):
    """E4M3 codes and inverse scales against the fp32 definition (scale = 448 / amax, round to
    nearest even, saturate). The hardware conversion (cvt.rn.satfinite.e4m3x2.f32) rounds a
    product lying within a few fp32 ulps above or below an E4M3 tie as the tie itself, so a
    small fraction of codes may sit one E4M3 step from the correctly rounded value."""
    from torchtitan_b200.ops._ext import ext

    torch.manual_seed(1)
    x = (torch.randn(300, 200, device="cuda") * torch.logspace(-2, 2, 200, device="cuda")).bfloat16()
    codes, inv = ext().f8_quantize(x, rowwise)
    assert codes.shape == (300, 256) and not codes[:, 200:].any()
    xf = x.float()
    amax = xf.abs().amax(-1, keepdim=True) if rowwise else xf.abs().amax()
    scale = 448.0 / amax.clamp_min(1e-12)
    ref = (xf * scale).clamp(-448, 448).to(torch.float8_e4m3fn).view(torch.uint8).int()
    got = codes[:, :200].int()
    torch.testing.assert_close(inv.view(-1), (1.0 / scale).view(-1), rtol=2e-7, atol=0)
    assert torch.equal(got >> 7, ref >> 7)                      # signs
    step = ((got & 0x7F) - (ref & 0x7F)).abs()                  # magnitudes are monotone codes
    assert int(step.max()) <= 1 and float((step > 0).float().mean()) < 5e-3, float((step > 0).float().mean())


@pytest.mark.parametrize("recipe", ["tensorwise", "rowwise", "rowwise_with_gw_hp"])
def test_float8_linear_kernel_path_matches_fake_quant(monkeypatch, recipe):
    """Forward and both backward GEMMs of the Float8 linear on the E4M3 tensor-core kernel
    against the quantize-dequantize emulation on the bf16 GEMM."""
    from torchtitan_b200.components.quantization.float8 import _F8LinearFn
    from torchtitan_b200.ops._ext import ext

    torch.manual_seed(4)
    x = torch.randn(2, 192, 512, device="cuda", dtype=torch.bfloat16)
    w = (torch.randn(640, 512, device="cuda") * 0.05).bfloat16()
    dy = torch.randn(2, 192, 640, device="cuda", dtype=torch.bfloat16)
    res = {}
    for flag in ("0", "1"):
        monkeypatch.setenv("TTB_FLOAT8_KERNEL", flag)
        xx, ww = x.clone().requires_grad_(), w.clone().requires_grad_()
        y = _F8LinearFn.apply(xx, ww, recipe)
        y.backward(dy)
        res[flag] = (y.detach().float(), xx.grad.float(), ww.grad.float())
    torch.cuda.synchronize()
    assert ext().mxgemm_error_code(True) == 0
    # relative error of the whole tensor: the kernel multiplies exact E4M3 products, the emulation
    # rounds the dequantized operands to bf16 first; both sit ~1e-2 from each other at K = 512
    for a, b in zip(res["1"], res["0"]):
        assert float((a - b).norm() / b.norm()) < 2e-2


@pytest.mark.parametrize("tile_n", [128, 256])
def test_mx_gemm_grouped_rows_matches_dequantized_product(tile_n):
    """Grouped-rows mode: every 128-row tile of A against its group's rows of the stacked B
    (a skipped tile, an empty group and the last group included) vs the CPU dequantized product."""
    from torchtitan_b200.ops._ext import ext
    from torchtitan_b200.ops.mx_gemm import mx_gemm_grouped, mx_quantize

    torch.manual_seed(0)
    G, n, K = 3, 256, 384
    P = 128 * 6
    tg = torch.tensor([0, 0, 2, -1, 2, 1], dtype=torch.int32, device="cuda")
    a = torch.randn(P, K, device="cuda").bfloat16()
    b = torch.randn(G * n, K, device="cuda").bfloat16()
    qa, sa = mx_quantize(a)
    qb, sb = mx_quantize(b)
    got = ext().gemm_mxfp8_grouped(qa, sa, qb, sb, tg, n, tile_n).float().cpu()
    want = mx_gemm_grouped(qa.cpu(), sa.cpu(), qb.cpu(), sb.cpu(), tg.cpu(), n).float()
    keep = (tg.cpu() >= 0).repeat_interleave(128)
    err = (got[keep] - want[keep]).norm() / want[keep].norm()
    assert err < 1e-2, err


def test_mxfp8_grouped_experts_kernel_path():
    """MXFP8 routed SwiGLU on the grouped block-scaled kernel: forward against the same
    quantized operands on the bf16 grouped GEMM; input and weight gradients against fp32."""
    from torchtitan_b200 import ops
    from torchtitan_b200.ops.grouped import mx_grouped_swiglu_cuda
    from torchtitan_b200.ops.quant import mx_fake_quant

    torch.manual_seed(0)
    E, D, H = 4, 256, 512
    counts = torch.tensor([300, 0, 517, 183], device="cuda")
    n = int(counts.sum())
    x = (torch.randn(n, D, device="cuda") * 0.5).bfloat16().requires_grad_()
    w1, w3 = ((torch.randn(E, H, D, device="cuda") * 0.05).bfloat16().requires_grad_() for _ in range(2))
    w2 = (torch.randn(E, D, H, device="cuda") * 0.05).bfloat16().requires_grad_()
    y = mx_grouped_swiglu_cuda(x, w1, w2, w3, counts)
    with torch.no_grad():
        want = ops.grouped_swiglu(mx_fake_quant(x, -1), mx_fake_quant(w1, -1), mx_fake_quant(w2, -1),
                                  mx_fake_quant(w3, -1), counts)
    assert (y.float() - want.float()).norm() / want.float().norm() < 3e-2
    g = torch.randn_like(y)
    y.backward(g)
    # fp32 reference of the unquantized experts
    xs, ws = x.detach().float().requires_grad_(), [w.detach().float().requires_grad_() for w in (w1, w2, w3)]
    outs, o = [], 0
    for e, c in enumerate(counts.tolist()):
        h = torch.nn.functional.silu(xs[o:o + c] @ ws[0][e].t()) * (xs[o:o + c] @ ws[2][e].t())
        outs.append(h @ ws[1][e].t())
        o += c
    torch.cat(outs).backward(g.float())
    for got, ref in ((x.grad, xs.grad), (w1.grad, ws[0].grad), (w2.grad, ws[1].grad), (w3.grad, ws[2].grad)):
        err = (got.float() - ref).norm() / ref.norm()
        assert err < 0.1, err
