"""Numerical parity with the Hugging Face ``transformers`` implementations: the
debug models are converted with each family's state-dict adapter, loaded into
the HF model, and both are run on the same tokens (CPU, fp32)."""
import re

import pytest
import torch

transformers = pytest.importorskip("transformers")


def _ours(module, flavor, **overrides):
    import importlib

    spec = importlib.import_module(f"torchtitan_b200.models.{module}").model_registry(flavor)
    for k, v in overrides.items():
        setattr(spec.model, k, v)
    torch.manual_seed(0)
    m = spec.model.build()
    m.init_weights()
    with torch.no_grad():  # exercise biases / correction terms that init to zero
        for n, p in m.named_buffers():
            if n.endswith("expert_bias"):
                p.normal_(0, 0.1)
        for n, p in m.named_parameters():
            if n.endswith(".bias") or n.endswith("sinks"):
                p.normal_(0, 0.1)
    m.eval()
    sd = spec.state_dict_adapter(spec.model, None).to_hf({k: v.detach() for k, v in m.state_dict().items()})
    return spec.model, m, sd


def _fuse_experts(sd):
    """HF checkpoints list experts one by one; the in-memory HF modules stack them."""
    fused = {}
    for k in list(sd):
        mm = re.fullmatch(r"(model\.layers\.\d+\.mlp\.experts)\.(\d+)\.(gate_proj|up_proj|down_proj)\.weight", k)
        if mm:
            fused.setdefault(mm.group(1), {}).setdefault(mm.group(3), {})[int(mm.group(2))] = sd.pop(k)
    for pre, d in fused.items():
        E = len(d["gate_proj"])
        sd[pre + ".gate_up_proj"] = torch.stack([torch.cat([d["gate_proj"][e], d["up_proj"][e]]) for e in range(E)])
        sd[pre + ".down_proj"] = torch.stack([d["down_proj"][e] for e in range(E)])
    return sd


def _compare(ours, hf, sd, vocab, seq=96, tol=1e-5):
    res = hf.load_state_dict(sd, strict=False)
    assert not res.missing_keys and not res.unexpected_keys, res
    hf.eval()
    tok = torch.randint(0, vocab, (2, seq), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        ref = hf(tok).logits
        out = ours(tok)
    assert float((ref - out).abs().max()) <= tol * float(ref.abs().max()), float((ref - out).abs().max())


def test_llama3_matches_hf():
    a, m, sd = _ours("llama3", "debugmodel")
    cfg = transformers.LlamaConfig(
        vocab_size=a.vocab_size, hidden_size=a.dim, intermediate_size=m.layers["0"].feed_forward.w1.weight.shape[0],
        num_hidden_layers=a.n_layers, num_attention_heads=a.n_heads, num_key_value_heads=a.n_kv_heads,
        rms_norm_eps=a.norm_eps, max_position_embeddings=a.max_seq_len, tie_word_embeddings=False,
        rope_parameters={"rope_type": "llama3", "rope_theta": a.rope_theta, "factor": a.rope_scaling_factor,
                         "low_freq_factor": 1.0, "high_freq_factor": 4.0, "original_max_position_embeddings": 8192})
    _compare(m, transformers.LlamaForCausalLM(cfg), sd, a.vocab_size)


@pytest.mark.parametrize("flavor", ["debugmodel", "debugmodel_moe"])
def test_qwen3_matches_hf(flavor):
    a, m, sd = _ours("qwen3", flavor)
    kw = dict(vocab_size=a.vocab_size, hidden_size=a.dim, intermediate_size=a.hidden_dim,
              num_hidden_layers=a.n_layers, num_attention_heads=a.n_heads, num_key_value_heads=a.n_kv_heads,
              head_dim=a.head_dim, rms_norm_eps=a.norm_eps, max_position_embeddings=a.max_seq_len,
              tie_word_embeddings=a.enable_weight_tying,
              rope_parameters={"rope_type": "default", "rope_theta": a.rope_theta})
    if a.moe_enabled:
        # the aux-loss-free expert bias has no HF counterpart: keep it zero here
        for mod in m.modules():
            if getattr(mod, "expert_bias", None) is not None:
                mod.expert_bias.zero_()
        cfg = transformers.Qwen3MoeConfig(**kw, num_experts=a.num_experts, num_experts_per_tok=a.top_k,
                                          moe_intermediate_size=a.moe_hidden_dim, norm_topk_prob=a.route_norm,
                                          decoder_sparse_step=a.decoder_sparse_step, mlp_only_layers=[])
        _compare(m, transformers.Qwen3MoeForCausalLM(cfg), _fuse_experts(sd), a.vocab_size)
    else:
        _compare(m, transformers.Qwen3ForCausalLM(transformers.Qwen3Config(**kw)), sd, a.vocab_size)


@pytest.mark.parametrize("yarn", [False, True])
def test_deepseek_v3_matches_hf(yarn):
    a, m, sd = _ours("deepseek_v3", "debugmodel_qlora", **({"max_seq_len": 16384} if yarn else {}))
    rope = ({"rope_type": "yarn", "rope_theta": a.rope_theta, "factor": a.rope_factor,
             "original_max_position_embeddings": a.original_seq_len, "beta_fast": a.beta_fast,
             "beta_slow": a.beta_slow, "mscale": a.mscale, "mscale_all_dim": a.mscale} if yarn
            else {"rope_type": "default", "rope_theta": a.rope_theta})
    cfg = transformers.DeepseekV3Config(
        vocab_size=a.vocab_size, hidden_size=a.dim, intermediate_size=a.inter_dim,
        moe_intermediate_size=a.moe_inter_dim, num_hidden_layers=a.n_layers, num_attention_heads=a.n_heads,
        num_key_value_heads=a.n_heads, n_shared_experts=a.n_shared_experts, n_routed_experts=a.n_routed_experts,
        routed_scaling_factor=a.route_scale, kv_lora_rank=a.kv_lora_rank, q_lora_rank=a.q_lora_rank,
        qk_rope_head_dim=a.qk_rope_head_dim, v_head_dim=a.v_head_dim, qk_nope_head_dim=a.qk_nope_head_dim,
        n_group=a.n_expert_groups, topk_group=a.n_limited_groups, num_experts_per_tok=a.n_activated_experts,
        first_k_dense_replace=a.n_dense_layers, norm_topk_prob=a.route_norm, rms_norm_eps=a.norm_eps,
        max_position_embeddings=a.max_seq_len, tie_word_embeddings=False, rope_interleave=True,
        rope_parameters=rope)
    _compare(m, transformers.DeepseekV3ForCausalLM(cfg), _fuse_experts(sd), a.vocab_size, tol=1e-4)


@pytest.mark.parametrize("yarn", [False, True])
def test_gpt_oss_matches_hf(yarn):
    a, m, sd = _ours("gpt_oss", "debugmodel", **({"max_seq_len": 131072} if yarn else {}))
    kw = {} if yarn else {"rope_parameters": {"rope_type": "default", "rope_theta": a.rope_theta}}
    cfg = transformers.GptOssConfig(
        vocab_size=a.vocab_size, hidden_size=a.dim, intermediate_size=a.moe_inter_dim, num_hidden_layers=a.n_layers,
        num_attention_heads=a.n_heads, num_key_value_heads=a.n_kv_heads, head_dim=a.head_dim,
        num_local_experts=a.num_experts, num_experts_per_tok=a.top_k, sliding_window=a.sliding_window,
        rms_norm_eps=a.norm_eps, tie_word_embeddings=False,
        layer_types=["sliding_attention" if i % 2 == 0 else "full_attention" for i in range(a.n_layers)], **kw)
    _compare(m, transformers.GptOssForCausalLM(cfg), sd, a.vocab_size, seq=200)  # 200 > sliding window


def test_llama4_matches_hf():
    a, m, sd = _ours("llama4", "debugmodel")
    for mod in m.modules():
        if getattr(mod, "expert_bias", None) is not None:
            mod.expert_bias.zero_()  # no HF counterpart
    hidden = m.layers["0"].feed_forward.w1.weight.shape[0]
    cfg = transformers.Llama4TextConfig(
        vocab_size=a.vocab_size, hidden_size=a.dim, intermediate_size=hidden, intermediate_size_mlp=hidden,
        num_hidden_layers=a.n_layers, num_attention_heads=a.n_heads, num_key_value_heads=a.n_kv_heads,
        head_dim=a.dim // a.n_heads, num_local_experts=a.num_experts, num_experts_per_tok=a.top_k,
        interleave_moe_layer_step=a.interleave_moe_layer_step, rms_norm_eps=a.norm_eps,
        attention_chunk_size=a.fixed_attn_block_size, use_qk_norm=a.use_qk_norm,
        attn_temperature_tuning=a.attn_temperature_tuning, floor_scale=int(a.floor_scale), attn_scale=a.attn_scale,
        max_position_embeddings=a.max_seq_len, tie_word_embeddings=False,
        rope_parameters={"rope_type": "llama3", "rope_theta": a.rope_theta, "factor": a.rope_scaling_factor,
                         "low_freq_factor": 1.0, "high_freq_factor": 4.0, "original_max_position_embeddings": 8192})
    _compare(m, transformers.Llama4ForCausalLM(cfg), sd, a.vocab_size, seq=512)  # 2 attention chunks


def _qwen3_vl_pair(**overrides):
    a, m, sd = _ours("qwen3_vl", "debugmodel", **overrides)
    vc = dict(depth=a.vision_layers, hidden_size=a.vision_dim, intermediate_size=a.vision_ffn_dim,
              num_heads=a.vision_heads, patch_size=a.patch_size, temporal_patch_size=a.temporal_patch_size,
              spatial_merge_size=a.spatial_merge_size, out_hidden_size=a.dim,
              num_position_embeddings=a.num_position_embeddings,
              deepstack_visual_indexes=list(a.deepstack_indices), hidden_act="gelu_pytorch_tanh")
    tc = dict(vocab_size=a.vocab_size, hidden_size=a.dim, intermediate_size=a.hidden_dim,
              num_hidden_layers=a.n_layers, num_attention_heads=a.n_heads, num_key_value_heads=a.n_kv_heads,
              head_dim=a.head_dim, rms_norm_eps=a.norm_eps, max_position_embeddings=a.max_seq_len,
              rope_parameters={"rope_type": "default", "rope_theta": a.rope_theta,
                               "mrope_section": list(a.mrope_section)})
    cfg = transformers.Qwen3VLConfig(vision_config=vc, text_config=tc, image_token_id=a.image_token_id,
                                     video_token_id=a.video_token_id, tie_word_embeddings=False)
    hf = transformers.Qwen3VLForConditionalGeneration(cfg)
    res = hf.load_state_dict(sd, strict=False)
    assert not res.missing_keys and not res.unexpected_keys, res
    return a, m, hf.eval()


def test_qwen3_vl_matches_hf():
    from torchtitan_b200.components.mm_dataloader import patchify

    a, m, hf = _qwen3_vl_pair()
    g = torch.Generator().manual_seed(1)
    # two images (4x6 and 2x2 merged tokens) in row 0, one (2x4) in row 1
    shapes = [(128, 192), (64, 64), (64, 128)]
    pix, grids = [], []
    for H, W in shapes:
        p, grid = patchify(torch.randn(3, H, W, generator=g), a.patch_size, a.temporal_patch_size,
                           a.spatial_merge_size)
        pix.append(p)
        grids.append(grid)
    S = 80
    tok = torch.randint(0, 2000, (2, S), generator=g)
    img = a.image_token_id
    tok[0, 5:5 + 24] = img
    tok[0, 40:44] = img
    tok[1, 10:18] = img
    pixel_values, grid_thw = torch.cat(pix), torch.tensor(grids)
    mm = (tok == img).int()
    with torch.no_grad():
        ref = hf(input_ids=tok, pixel_values=pixel_values, image_grid_thw=grid_thw, mm_token_type_ids=mm).logits
        out = m(tok, pixel_values=pixel_values, grid_thw=grid_thw)
    err = float((ref - out).abs().max())
    assert err <= 2e-5 * float(ref.abs().max()), err
    # text only
    t2 = torch.randint(0, 2000, (2, 32), generator=g)
    with torch.no_grad():
        assert torch.allclose(hf(input_ids=t2).logits, m(t2), atol=1e-4)


def test_qwen3_vl_state_dict_roundtrip():
    from torchtitan_b200.models.qwen3_vl import model_registry

    spec = model_registry("debugmodel")
    torch.manual_seed(0)
    m = spec.model.build()
    m.init_weights()
    ad = spec.state_dict_adapter(spec.model, None)
    sd = {k: v.detach() for k, v in m.state_dict().items()}
    back = ad.from_hf(ad.to_hf(sd))
    assert set(back) == set(sd)
    assert all(torch.equal(back[k], sd[k]) for k in sd)


def test_siglip2_encoder_matches_hf():
    """The VLM's SigLIP2 encoder on two images of different aspect ratios (padded batch)."""
    from torchtitan_b200.components.mm_dataloader import patchify_raster

    a, m, sd = _ours("vlm", "debugmodel")
    cfg = transformers.Siglip2VisionConfig(hidden_size=a.vit_dim, intermediate_size=a.vit_ffn_dim,
                                           num_hidden_layers=a.vit_layers, num_attention_heads=a.vit_heads,
                                           num_channels=a.channels, patch_size=a.patch_size,
                                           num_patches=a.n_pos_embs ** 2, layer_norm_eps=a.vit_eps,
                                           hidden_act="gelu_pytorch_tanh", vision_use_head=False)
    hf = transformers.Siglip2VisionModel(cfg).eval()
    vsd = {k[len("vision_model."):]: v for k, v in sd.items() if k.startswith("vision_model.")}
    res = hf.vision_model.load_state_dict(vsd, strict=False)
    assert not res.missing_keys and not res.unexpected_keys, res
    g = torch.Generator().manual_seed(2)
    p1, g1 = patchify_raster(torch.randn(3, 96, 160, generator=g), a.patch_size)   # 6 x 10
    p2, g2 = patchify_raster(torch.randn(3, 128, 64, generator=g), a.patch_size)   # 8 x 4
    L = 64
    pix = torch.zeros(2, L, p1.shape[1])
    pix[0, :60], pix[1, :32] = p1, p2
    mask = torch.zeros(2, L, dtype=torch.long)
    mask[0, :60], mask[1, :32] = 1, 1
    shapes = torch.tensor([g1, g2])
    with torch.no_grad():
        ref = hf(pixel_values=pix, pixel_attention_mask=mask, spatial_shapes=shapes).last_hidden_state
        out = m.encoder(pix, shapes)
    want = torch.cat([ref[0, :60], ref[1, :32]])
    assert float((want - out).abs().max()) <= 2e-5 * float(want.abs().max()), float((want - out).abs().max())


def test_vlm_state_dict_round_trip():
    from torchtitan_b200.models.vlm import model_registry

    spec = model_registry("debugmodel")
    torch.manual_seed(0)
    m = spec.model.build()
    m.init_weights()
    ad = spec.state_dict_adapter(spec.model, None)
    sd = {k: v.detach() for k, v in m.state_dict().items()}
    back = ad.from_hf(ad.to_hf(sd))
    assert set(back) == set(sd) and all(torch.equal(back[k], sd[k]) for k in sd)
