"""The Qwen3 / DeepSeek-V3 / Llama 4 / GPT-OSS / Kimi-Linear debug models on a B200: one
bf16 forward+backward through the sm_100a kernels, compared with the same weights run in
fp32 PyTorch on the CPU (logits, loss, parameter gradients)."""
import importlib

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


# Tolerances: dense models stay within bf16 rounding; in MoE models a near-tied top-k choice
# can flip between bf16 and fp32 at random init, which moves whole tokens to other experts
# (measured on the CPU alone: Kimi-Linear logits 0.13 relative error, all of it entering at the
# first MoE layer), so their logits and router/expert gradients get a wider bound.
@pytest.mark.parametrize("module,flavor,logit_tol,grad_tol", [
    ("qwen3", "debugmodel", 3e-2, 0.1), ("qwen3", "debugmodel_moe", 0.2, 0.4),
    ("deepseek_v3", "debugmodel", 0.2, 0.4), ("llama4", "debugmodel", 0.2, 0.4),
    ("gpt_oss", "debugmodel", 0.2, 0.4), ("kimi_linear", "debugmodel", 0.25, 0.5),
    ("kimi_linear", "debugmodel_block_attn_res", 0.25, 0.5)])
def test_family_bf16_forward_backward(module, flavor, logit_tol, grad_tol):
    """bf16 on the kernels vs the same weights in fp32 PyTorch on the CPU: logits, loss and
    every parameter gradient (relative L2 error)."""
    spec = importlib.import_module(f"torchtitan_b200.models.{module}").model_registry(flavor)
    torch.manual_seed(0)
    ref = spec.model.build()
    ref.init_weights()
    with torch.device("cuda"):
        model = spec.model.build()
    model.init_weights(buffer_device=torch.device("cuda"))
    model.load_state_dict(ref.state_dict())
    for p in model.parameters():
        p.data = p.data.bfloat16()
    tokens = torch.randint(0, spec.model.vocab_size, (1, 512))
    labels = tokens.roll(-1, 1).flatten()
    want = ref(tokens)
    want_loss = F.cross_entropy(want.flatten(0, 1), labels)
    want_loss.backward()
    logits = model(tokens.cuda())
    loss = F.cross_entropy(logits.flatten(0, 1).float(), labels.cuda())
    loss.backward()
    rel = float((logits.float().cpu() - want.detach()).norm() / want.detach().norm())
    assert rel < logit_tol, rel
    assert abs(float(loss) - float(want_loss)) < 2e-2 * float(want_loss)
    named_ref = dict(ref.named_parameters())
    worst = []
    for n, p in model.named_parameters():
        r = named_ref[n].grad
        if r is None or r.norm() == 0:
            continue
        assert p.grad is not None and torch.isfinite(p.grad).all(), n
        if p.numel() < 64:  # per-head scalars (e.g. KDA's A_log): sums of many cancelling terms,
            continue        # checked against PyTorch by the kernel tests instead
        worst.append((float((p.grad.float().cpu() - r).norm() / r.norm()), n))
    worst.sort(reverse=True)
    assert worst[0][0] < grad_tol, worst[:3]


def test_qwen3_vl_bf16_forward_backward_with_images():
    """Vision encoder (per-frame bidirectional flash attention, 2-D rotary) + MRoPE decoder
    with DeepStack, bf16 on the kernels, against the same model in fp32 PyTorch on the CPU."""
    from torchtitan_b200.components.mm_dataloader import patchify

    spec = importlib.import_module("torchtitan_b200.models.qwen3_vl").model_registry("debugmodel")
    a = spec.model
    torch.manual_seed(0)
    ref = a.build()
    ref.init_weights()
    with torch.device("cuda"):
        model = a.build()
    model.load_state_dict(ref.state_dict())
    model.rope.init_weights(torch.device("cuda"))
    model.vision_encoder.init_buffers(torch.device("cuda"))
    model.mrope_axis = ref.mrope_axis.cuda()
    for p in model.parameters():
        p.data = p.data.bfloat16()
    g = torch.Generator().manual_seed(1)
    pix, grids = zip(*[patchify(torch.randn(3, 256, 256, generator=g), a.patch_size, a.temporal_patch_size,
                                a.spatial_merge_size) for _ in range(2)])
    tokens = torch.randint(0, 2000, (1, 512), generator=g)
    tokens[0, 10:74] = a.image_token_id
    tokens[0, 300:364] = a.image_token_id
    kw = dict(pixel_values=torch.cat(pix), grid_thw=torch.tensor(grids))
    with torch.no_grad():
        want = ref(tokens, **kw)
    logits = model(tokens.cuda(), pixel_values=kw["pixel_values"].cuda().bfloat16(), grid_thw=kw["grid_thw"])
    rel = float((logits.float().cpu() - want).norm() / want.norm())
    assert rel < 3e-2, rel
    loss = F.cross_entropy(logits.flatten(0, 1).float(), tokens.cuda().roll(-1, 1).flatten())
    loss.backward()
    assert torch.isfinite(loss)
    assert all(p.grad is not None and torch.isfinite(p.grad).all() for p in model.parameters())


def test_flux_bf16_forward_backward():
    """FLUX double/single stream blocks on the kernels (bidirectional flash attention with
    per-row 3-axis RoPE tables, RMSNorm q/k) against fp32 PyTorch on the CPU."""
    from torchtitan_b200.models.flux.model import FluxModelArgs
    from torchtitan_b200.models.flux.sampling import latent_position_ids, pack_latents, text_position_ids

    a = FluxModelArgs(hidden_size=256, num_heads=2, depth=2, depth_single_blocks=2, context_in_dim=64,
                      vec_in_dim=32)
    torch.manual_seed(0)
    ref = a.build()
    ref.init_weights()
    with torch.no_grad():
        for p in ref.parameters():
            p.add_(torch.randn_like(p) * 0.05)
    with torch.device("cuda"):
        model = a.build()
    model.load_state_dict(ref.state_dict())
    for p in model.parameters():
        p.data = p.data.bfloat16()
    g = torch.Generator().manual_seed(1)
    B, h, w = 2, 32, 32
    inp = dict(img=pack_latents(torch.randn(B, 16, h, w, generator=g)), img_ids=latent_position_ids(B, h, w),
               txt=torch.randn(B, 64, 64, generator=g), txt_ids=text_position_ids(B, 64),
               timesteps=torch.rand(B, generator=g), y=torch.randn(B, 32, generator=g))
    with torch.no_grad():
        want = ref(**inp)
    out = model(**{k: v.cuda() for k, v in inp.items()})
    rel = float((out.float().cpu() - want).norm() / want.norm())
    assert rel < 3e-2, rel
    out.float().pow(2).mean().backward()
    assert all(p.grad is not None and torch.isfinite(p.grad).all() for p in model.parameters())


def test_vlm_bf16_forward_backward_with_images():
    """Llama 3 + SigLIP2 (per-image bidirectional flash attention over unpadded patches)
    against the same model in fp32 PyTorch on the CPU."""
    from torchtitan_b200.components.mm_dataloader import patchify_raster

    spec = importlib.import_module("torchtitan_b200.models.vlm").model_registry("debugmodel")
    a = spec.model
    torch.manual_seed(0)
    ref = a.build()
    ref.init_weights()
    with torch.device("cuda"):
        model = a.build()
    model.load_state_dict(ref.state_dict())
    model.rope.init_weights(torch.device("cuda"))
    for p in model.parameters():
        p.data = p.data.bfloat16()
    g = torch.Generator().manual_seed(1)
    p1, g1 = patchify_raster(torch.randn(3, 128, 192, generator=g), a.patch_size)  # 8 x 12
    p2, g2 = patchify_raster(torch.randn(3, 64, 128, generator=g), a.patch_size)   # 4 x 8
    pix = torch.zeros(2, 96, p1.shape[1])
    pix[0, :96], pix[1, :32] = p1, p2
    tokens = torch.randint(0, 2000, (1, 512), generator=g)
    tokens[0, 20:116] = a.image_token_id
    tokens[0, 300:332] = a.image_token_id
    grid = torch.tensor([g1, g2])
    with torch.no_grad():
        want = ref(tokens, pixel_values=pix, grid_hw=grid)
    logits = model(tokens.cuda(), pixel_values=pix.cuda().bfloat16(), grid_hw=grid)
    rel = float((logits.float().cpu() - want).norm() / want.norm())
    assert rel < 3e-2, rel
    loss = F.cross_entropy(logits.flatten(0, 1).float(), tokens.cuda().roll(-1, 1).flatten())
    loss.backward()
    assert all(p.grad is not None and torch.isfinite(p.grad).all() for p in model.parameters())


def test_gpt_oss_chunked_sliding_window_on_flash_kernel():
    from torchtitan_b200.models.gpt_oss.model import sink_attention, sliding_window_attention_lse

    torch.manual_seed(0)
    q = torch.randn(2, 1000, 8, 64, device="cuda", dtype=torch.bfloat16)
    k, v = (torch.randn(2, 1000, 2, 64, device="cuda", dtype=torch.bfloat16) for _ in range(2))
    sinks = torch.randn(8, device="cuda")
    o, lse = sliding_window_attention_lse(q, k, v, 128, 0.125)
    out = o.float() * torch.sigmoid(lse - sinks.view(1, 1, -1))[..., None]
    ref = sink_attention(q.float(), k.float(), v.float(), sinks, 128, 0.125)
    assert float((out - ref).norm() / ref.norm()) < 2e-2
