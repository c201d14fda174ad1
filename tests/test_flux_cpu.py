"""FLUX (reference ``models/flux``): the transformer against an independent
formulation of the published FLUX.1 blocks (rotation-matrix RoPE, head-major SDPA),
latent packing and the sampling schedule, the diffusers name mapping, the
autoencoder, and the trainer end to end on CPU."""
import math

import pytest
import torch
import torch.nn.functional as F

from torchtitan_b200.models.flux import model_registry
from torchtitan_b200.models.flux.model import FluxModelArgs, timestep_embedding
from torchtitan_b200.models.flux.sampling import (get_schedule, latent_position_ids, pack_latents,
                                                  text_position_ids, unpack_latents)

SMALL = dict(hidden_size=256, num_heads=2, depth=2, depth_single_blocks=2, context_in_dim=64, vec_in_dim=32,
             axes_dim=(16, 56, 56))


def _model(**kw):
    torch.manual_seed(0)
    m = FluxModelArgs(**{**SMALL, **kw}).build()
    m.init_weights()
    with torch.no_grad():  # zero-initialised modulations would hide most of the math
        for p in m.parameters():
            p.add_(torch.randn_like(p) * 0.05)
    return m


def _rope_mats(ids, axes, theta):
    mats = []
    for i, d in enumerate(axes):
        w = 1.0 / theta ** (torch.arange(0, d, 2, dtype=torch.float64) / d)
        a = ids[..., i].double()[..., None] * w
        mats.append(torch.stack([a.cos(), -a.sin(), a.sin(), a.cos()], -1).view(*a.shape, 2, 2))
    return torch.cat(mats, -3).float()[:, None]  # [B, 1, L, D/2, 2, 2]


def _apply(x, pe):  # x [B, H, L, D]
    x2 = x.float().reshape(*x.shape[:-1], -1, 1, 2)
    return (pe[..., 0] * x2[..., 0] + pe[..., 1] * x2[..., 1]).reshape(x.shape)


def _ref_forward(m, img, img_ids, txt, txt_ids, t, y):
    a = m.model_args
    H = a.num_heads
    pe = _rope_mats(torch.cat([txt_ids, img_ids], 1), a.axes_dim, a.theta)
    ln = lambda x: F.layer_norm(x, x.shape[-1:], eps=1e-6)
    rms = lambda x, w: x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * w
    lin = lambda l, x: F.linear(x, l.weight, l.bias)

    def heads(x):
        B, L, D = x.shape
        return x.view(B, L, 3, H, -1).permute(2, 0, 3, 1, 4)

    def attn(q, k, v):
        q, k = _apply(q, pe), _apply(k, pe)
        o = F.scaled_dot_product_attention(q, k, v)
        return o.permute(0, 2, 1, 3).flatten(2)

    img = lin(m.img_in, img)
    vec = lin(m.time_in.out_layer, F.silu(lin(m.time_in.in_layer, timestep_embedding(t, 256))))
    vec = vec + lin(m.vector_in.out_layer, F.silu(lin(m.vector_in.in_layer, y)))
    txt = lin(m.txt_in, txt)
    for b in m.double_blocks:
        im = lin(b.img_mod.lin, F.silu(vec))[:, None].chunk(6, -1)
        tm = lin(b.txt_mod.lin, F.silu(vec))[:, None].chunk(6, -1)
        iq, ik, iv = heads(lin(b.img_attn.qkv, (1 + im[1]) * ln(img) + im[0]))
        tq, tk, tv = heads(lin(b.txt_attn.qkv, (1 + tm[1]) * ln(txt) + tm[0]))
        iq, ik = rms(iq, b.img_attn.norm.query_norm.weight), rms(ik, b.img_attn.norm.key_norm.weight)
        tq, tk = rms(tq, b.txt_attn.norm.query_norm.weight), rms(tk, b.txt_attn.norm.key_norm.weight)
        o = attn(torch.cat([tq, iq], 2), torch.cat([tk, ik], 2), torch.cat([tv, iv], 2))
        to, io = o[:, :txt.shape[1]], o[:, txt.shape[1]:]
        img = img + im[2] * lin(b.img_attn.proj, io)
        x = (1 + im[4]) * ln(img) + im[3]
        img = img + im[5] * lin(b.img_mlp.fc2, F.gelu(lin(b.img_mlp.fc1, x), approximate="tanh"))
        txt = txt + tm[2] * lin(b.txt_attn.proj, to)
        x = (1 + tm[4]) * ln(txt) + tm[3]
        txt = txt + tm[5] * lin(b.txt_mlp.fc2, F.gelu(lin(b.txt_mlp.fc1, x), approximate="tanh"))
    x = torch.cat([txt, img], 1)
    h = a.hidden_size
    for b in m.single_blocks:
        sh, sc, g = lin(b.modulation.lin, F.silu(vec))[:, None].chunk(3, -1)
        qkv, mlp = lin(b.linear1, (1 + sc) * ln(x) + sh).split([3 * h, b.mlp], -1)
        q, k, v = heads(qkv)
        q, k = rms(q, b.norm.query_norm.weight), rms(k, b.norm.key_norm.weight)
        o = attn(q, k, v)
        x = x + g * lin(b.linear2, torch.cat([o, F.gelu(mlp, approximate="tanh")], -1))
    x = x[:, txt.shape[1]:]
    sh, sc = lin(m.final_layer.adaLN_modulation, F.silu(vec))[:, None].chunk(2, -1)
    return lin(m.final_layer.linear, (1 + sc) * ln(x) + sh)


def test_flux_matches_independent_formulation():
    m = _model()
    B, h, w = 2, 8, 12
    g = torch.Generator().manual_seed(0)
    lat = torch.randn(B, 16, h, w, generator=g)
    img, img_ids = pack_latents(lat), latent_position_ids(B, h, w)
    txt = torch.randn(B, 7, 64, generator=g)
    txt_ids = text_position_ids(B, 7)
    t, y = torch.rand(B, generator=g), torch.randn(B, 32, generator=g)
    with torch.no_grad():
        out = m(img, img_ids, txt, txt_ids, t, y)
        ref = _ref_forward(m, img, img_ids, txt, txt_ids, t, y)
    assert out.shape == (B, (h // 2) * (w // 2), 64)
    assert float((out - ref).abs().max()) < 1e-4 * float(ref.abs().max()) + 1e-6


def test_packing_and_schedule():
    x = torch.randn(2, 16, 6, 10)
    p = pack_latents(x)
    assert p.shape == (2, 15, 64) and torch.equal(unpack_latents(p, 6, 10), x)
    assert torch.equal(p[0, 1, :4], torch.stack([x[0, 0, 0, 2], x[0, 0, 0, 3], x[0, 0, 1, 2], x[0, 0, 1, 3]]))
    ids = latent_position_ids(1, 6, 10)
    assert ids[0, 7].tolist() == [0, 1, 2]
    s = get_schedule(10, 4096)
    assert s[0] == 1.0 and s[-1] == 0.0 and all(a > b for a, b in zip(s, s[1:]))
    u = get_schedule(10, 4096, shift=False)
    mu = 1.15
    assert abs(s[5] - math.exp(mu) / (math.exp(mu) + 1 / u[5] - 1)) < 1e-12 and s[5] > u[5]


def test_diffusers_name_round_trip():
    spec = model_registry("flux-debug")
    for k, v in SMALL.items():
        setattr(spec.model, k, v)
    m = _model()
    ad = spec.state_dict_adapter(spec.model, None)
    sd = m.state_dict()
    hf = ad.to_hf(sd)
    assert hf["transformer_blocks.0.attn.add_k_proj.weight"].shape == (256, 256)
    assert hf["single_transformer_blocks.1.proj_mlp.weight"].shape == (1024, 256)
    scale_shift = hf["norm_out.linear.weight"]
    assert torch.equal(scale_shift[:256], sd["final_layer.adaLN_modulation.weight"][256:])
    back = ad.from_hf(hf)
    assert set(back) == set(sd) and all(torch.equal(back[k], sd[k]) for k in sd)


def test_autoencoder_shapes_and_checkpoint_load(tmp_path):
    from safetensors.torch import save_file

    from torchtitan_b200.models.flux.autoencoder import build_autoencoder

    a = FluxModelArgs(ae_ch=32, ae_ch_mult=(1, 2), ae_num_res_blocks=1)
    ae = build_autoencoder(a, None, "cpu", torch.float32)
    x = torch.rand(2, 3, 32, 32) * 2 - 1
    z = ae.encode(x)
    assert z.shape == (2, 16, 16, 16)
    assert ae.decode(z).shape == x.shape
    p = tmp_path / "ae.safetensors"
    save_file({k: v.contiguous() for k, v in ae.state_dict().items()}, str(p))
    ae2 = build_autoencoder(a, str(p), "cpu", torch.float32)
    assert torch.equal(ae2.encode(x), z)


def _small_cfg(tmp_path, steps=3):
    from torchtitan_b200.models.flux.config_registry import flux_debugmodel

    cfg = flux_debugmodel()
    for k, v in SMALL.items():
        setattr(cfg.model_spec.model, k, v)
    a = cfg.model_spec.model
    a.ae_ch, a.ae_ch_mult, a.ae_num_res_blocks = 32, (1, 2, 2, 2), 1
    cfg.dataloader.img_size = 64
    cfg.encoder.max_t5_encoding_len = 8
    cfg.training.local_batch_size = 2
    cfg.training.steps = steps
    cfg.training.seq_len = 16 + 8
    cfg.training.dtype = cfg.training.mixed_precision_param = "float32"
    cfg.dump_folder = str(tmp_path)
    return cfg


def test_flux_trainer_steps_and_generates(tmp_path):
    from torchtitan_b200.models.flux.trainer import FluxTrainer

    t = FluxTrainer(_small_cfg(tmp_path))
    t.train()
    assert t.step == 3 and math.isfinite(float(t.last_loss))
    img = t.generate(["a red house"], size=64, steps=2, cfg_scale=3.0)
    assert img.shape == (1, 3, 64, 64) and torch.isfinite(img).all()
    t.close()
