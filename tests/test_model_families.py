"""CPU tests for the Qwen3, DeepSeek-V3, Llama 4, GPT-OSS and dense AttnRes families:
forward/backward, HF name mapping round trips, and the attention variants
against plain PyTorch formulations."""
import pytest
import torch
import torch.nn.functional as F

FAMILIES = [("qwen3", "debugmodel"), ("qwen3", "debugmodel_moe"), ("deepseek_v3", "debugmodel"),
            ("deepseek_v3", "debugmodel_qlora"), ("llama4", "debugmodel"), ("gpt_oss", "debugmodel"),
            ("attention_residual", "debugmodel"), ("attention_residual", "debugmodel_full"), ("qwen3_vl", "debugmodel"),
            ("vlm", "debugmodel")]


def _build(module, flavor, seq=64):
    import importlib

    spec = importlib.import_module(f"torchtitan_b200.models.{module}").model_registry(flavor)
    torch.manual_seed(0)
    model = spec.model.build()
    model.init_weights()
    return spec, model


@pytest.mark.parametrize("module,flavor", FAMILIES)
def test_forward_backward_and_flops(module, flavor):
    spec, model = _build(module, flavor)
    tokens = torch.randint(0, spec.model.vocab_size, (2, 64))
    logits = model(tokens)
    assert logits.shape == (2, 64, spec.model.vocab_size)
    loss = F.cross_entropy(logits.flatten(0, 1).float(), tokens.roll(-1, 1).flatten())
    assert torch.isfinite(loss) and 6.0 < float(loss) < 10.0
    loss.backward()
    missing = [n for n, p in model.named_parameters() if p.grad is None]
    assert not missing, missing
    n, flops = spec.model.get_nparams_and_flops(model, 64)
    assert n == sum(p.numel() for p in model.parameters()) and flops > 0
    # MoE families count only the routed experts a token uses
    dense_flops = 6 * (n - model.tok_embeddings.weight.numel())
    if any("experts" in name for name, _ in model.named_parameters()):
        assert flops < dense_flops + 6 * spec.model.n_layers * 2 * 10 ** 6


@pytest.mark.parametrize("module", ["qwen3", "deepseek_v3"])
def test_hf_adapter_round_trip(module):
    spec, model = _build(module, "debugmodel_moe" if module == "qwen3" else "debugmodel")
    sd = {k: v.detach() for k, v in model.state_dict().items()}
    adapter = spec.state_dict_adapter(spec.model, None)
    hf = adapter.to_hf(sd)
    assert any(".mlp.experts.0." in k for k in hf)
    back = adapter.from_hf(hf)
    for k, v in sd.items():
        if k.endswith("tokens_per_expert") or (module == "qwen3" and k.endswith("expert_bias")):
            continue
        assert k in back, k
        assert torch.equal(back[k], v), k


def test_qwen3_adapter_permutes_qk_norm_with_rows():
    from torchtitan_b200.models.qwen3.state_dict_adapter import Qwen3StateDictAdapter as Ad

    w = torch.arange(8.0)
    halves = Ad.interleaved_to_halves(w[:, None], 1)[:, 0]
    assert torch.equal(halves, torch.tensor([0., 2, 4, 6, 1, 3, 5, 7]))


def test_sink_attention_reduces_to_causal_softmax():
    from torchtitan_b200.models.gpt_oss.model import sink_attention

    torch.manual_seed(0)
    q, k, v = (torch.randn(1, 16, 4, 8) for _ in range(3))
    k2, v2 = k[:, :, :2], v[:, :, :2]
    sinks = torch.full((4,), -1e9)
    ref = F.scaled_dot_product_attention(q.transpose(1, 2), k2.repeat_interleave(2, 2).transpose(1, 2),
                                         v2.repeat_interleave(2, 2).transpose(1, 2), is_causal=True).transpose(1, 2)
    torch.testing.assert_close(sink_attention(q, k2, v2, sinks, 0, 8 ** -0.5), ref, rtol=1e-5, atol=1e-5)
    # a sink of logit s scales every row by 1 / (1 + exp(s - lse))
    sinks0 = torch.zeros(4)
    out = sink_attention(q, k, v, sinks0, 0, 8 ** -0.5)
    s = torch.einsum("bshd,bthd->bhst", q, k) * 8 ** -0.5
    s = s.masked_fill(~torch.ones(16, 16, dtype=torch.bool).tril(), float("-inf"))
    lse = torch.logsumexp(s, -1).transpose(1, 2)[..., None]
    full = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                          is_causal=True).transpose(1, 2)
    torch.testing.assert_close(out, full * torch.sigmoid(lse), rtol=1e-5, atol=1e-5)
    # window: query i sees keys i-w+1..i only
    w = sink_attention(q, k, v, sinks, 3, 8 ** -0.5)
    torch.testing.assert_close(w[:, 0], full[:, 0], rtol=1e-5, atol=1e-5)
    qi = 10
    sl = slice(qi - 2, qi + 1)
    ref_row = F.scaled_dot_product_attention(q[:, qi:qi + 1].transpose(1, 2), k[:, sl].transpose(1, 2),
                                             v[:, sl].transpose(1, 2)).transpose(1, 2)
    torch.testing.assert_close(w[:, qi:qi + 1], ref_row, rtol=1e-5, atol=1e-5)


def test_llama4_chunked_attention_is_block_causal():
    spec, model = _build("llama4", "debugmodel")
    att = model.layers["0"].attention
    assert att.use_rope and att.block == 256
    assert not model.layers["3"].attention.use_rope  # every 4th layer is NoPE
    att.block = 4
    torch.manual_seed(0)
    q, k, v = (torch.randn(1, 12, 16, 16) for _ in range(3))
    k, v = k[:, :, :8], v[:, :, :8]
    out = att.inner_attention(q, k, v)
    i = torch.arange(12)
    mask = (i[:, None] >= i[None, :]) & (i[:, None] // 4 == i[None, :] // 4)
    ref = F.scaled_dot_product_attention(q.transpose(1, 2), k.repeat_interleave(2, 2).transpose(1, 2),
                                         v.repeat_interleave(2, 2).transpose(1, 2), attn_mask=mask).transpose(1, 2)
    torch.testing.assert_close(out, ref, rtol=1e-4, atol=1e-4)
    # a sequence that is not a multiple of the chunk stays chunked (the last chunk is short)
    out = att.inner_attention(q[:, :10], k[:, :10], v[:, :10])
    torch.testing.assert_close(out, ref[:, :10], rtol=1e-4, atol=1e-4)


def test_deepseek_mla_scale_and_shared_rope_key():
    spec, model = _build("deepseek_v3", "debugmodel")
    a = spec.model
    assert a.softmax_scale == pytest.approx(192 ** -0.5)
    a.max_seq_len, a.original_seq_len = 16384, 4096
    m = 0.1 * a.mscale * torch.log(torch.tensor(a.rope_factor)).item() + 1
    assert a.softmax_scale == pytest.approx(192 ** -0.5 * m * m)
    blk = model.layers["1"]
    assert blk.moe_enabled and blk.moe.shared_experts is not None
    assert not model.layers["0"].moe_enabled


@pytest.mark.parametrize("module,config", [("qwen3", "qwen3_debugmodel_moe"), ("deepseek_v3", "deepseek_v3_debugmodel"),
                                           ("llama4", "llama4_debugmodel"), ("gpt_oss", "gpt_oss_debugmodel"),
                                           ("qwen3_vl", "qwen3_vl_debugmodel"), ("vlm", "vlm_debugmodel")])
def test_trainer_runs_family_configs(module, config, tmp_path):
    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.trainer import Trainer

    cfg = ConfigManager().parse_args(["--module", module, "--config", config, "--training.steps", "2",
                                      "--training.seq-len", "128", "--training.local-batch-size", "2",
                                      "--training.dtype", "float32", "--training.mixed-precision-param", "float32",
                                      "--activation-checkpoint.mode", "selective", "--dump-folder", str(tmp_path)])
    t = Trainer(cfg)
    t.train()
    assert t.step == 2
    assert torch.isfinite(torch.tensor(t.metrics_processor.last_metrics["loss_metrics/global_avg_loss"]))
    t.close()


def test_block_attn_res_uniform_at_init_and_softmax_weights():
    from torchtitan_b200.models.common import RMSNorm
    from torchtitan_b200.models.common.attn_res import block_attn_res

    torch.manual_seed(0)
    norm = RMSNorm(8)
    norm.init_weights()
    blocks = [torch.randn(2, 3, 8) for _ in range(3)]
    partial = torch.randn(2, 3, 8)
    out = block_attn_res(blocks, partial, torch.zeros(1, 8), norm)
    torch.testing.assert_close(out, torch.stack(blocks + [partial]).mean(0))
    q = torch.randn(1, 8)
    V = torch.stack(blocks + [partial])
    Kn = V * torch.rsqrt(V.pow(2).mean(-1, keepdim=True) + 1e-5)
    w = torch.softmax((Kn @ q[0]), 0)
    torch.testing.assert_close(block_attn_res(blocks, partial, q, norm), (w[..., None] * V).sum(0))


def test_kimi_multimodal_splices_projected_patches():
    from torchtitan_b200.models.kimi_linear import model_registry
    from torchtitan_b200.models.kimi_linear.multimodal import (KimiLinearMultimodal, PatchVisionTower,
                                                               image_label_mask)

    spec = model_registry("debugmodel")
    torch.manual_seed(0)
    llm = spec.model.build()
    tower = PatchVisionTower(image_size=28, patch=14, dim=32)
    mm = KimiLinearMultimodal(llm, vision_tower=tower, vision_dim=32, projector_dim=64)
    mm.init_weights()
    tokens = torch.randint(0, spec.model.vocab_size, (2, 64))
    tokens[0, 5:9] = -200   # one image = 4 patches per sample
    tokens[1, 20:24] = -200
    pix = torch.randn(2, 1, 3, 28, 28)
    emb = mm.embed(tokens, pix)
    proj = mm.projector(tower(pix.flatten(0, 1)))
    torch.testing.assert_close(emb[0, 5:9], proj[0])
    torch.testing.assert_close(emb[1, 20:24], proj[1])
    torch.testing.assert_close(emb[0, :5], llm.embed_tokens(tokens[0, :5]))
    logits = mm(tokens, pix)
    labels = image_label_mask(tokens.roll(-1, 1), tokens)
    loss = F.cross_entropy(logits.flatten(0, 1).float(), labels.flatten(), ignore_index=-100)
    loss.backward()
    assert mm.projector.fc1.weight.grad is not None and tower.proj.weight.grad is None
    assert (labels[0, 4:9] == -100).all()


@pytest.mark.parametrize("S,W", [(50, 8), (64, 16), (17, 16)])
def test_gpt_oss_chunked_sliding_window_matches_masked_softmax(S, W):
    """Sliding-window attention as two causal attentions per window chunk (lse merge, then the
    sink) equals the masked softmax with the sink column, values and gradients."""
    from torchtitan_b200.models.gpt_oss.model import sink_attention, sliding_window_attention_lse

    torch.manual_seed(0)
    q = torch.randn(2, S, 4, 16, requires_grad=True)
    k, v = (torch.randn(2, S, 2, 16, requires_grad=True) for _ in range(2))
    sinks = torch.randn(4)
    o, lse = sliding_window_attention_lse(q, k, v, W, 0.25)
    out = o * torch.sigmoid(lse - sinks.view(1, 1, -1))[..., None]
    ref = sink_attention(q, k, v, sinks, W, 0.25)
    assert torch.allclose(out, ref, atol=1e-5)
    g = torch.randn_like(ref)
    ga = torch.autograd.grad(out, (q, k, v), g)
    gb = torch.autograd.grad(ref, (q, k, v), g)
    for a, b in zip(ga, gb):
        assert torch.allclose(a, b, atol=1e-5)
