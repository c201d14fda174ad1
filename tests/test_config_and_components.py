"""CPU unit tests: config system, registry, parallel dims, LR schedule, data, optimizers, adapters."""
import dataclasses
import math

import pytest
import torch

from torchtitan_b200.components.dataloader import SyntheticDataLoader
from torchtitan_b200.components.lr_scheduler import wsd_factor
from torchtitan_b200.config import Configurable
from torchtitan_b200.config.manager import ConfigManager, split_module_and_config
from torchtitan_b200.parallel.parallel_dims import ParallelDims
from torchtitan_b200.parallel.pipeline import generate_llm_fqn_per_model_part


def test_configurable_requires_kw_only_slots():
    with pytest.raises(TypeError):
        class Bad(Configurable):
            @dataclasses.dataclass
            class Config(Configurable.Config):
                x: int = 1

    class Good(Configurable):
        @dataclasses.dataclass(kw_only=True, slots=True)
        class Config(Configurable.Config):
            x: int = 1

        def __init__(self, config, **kw):
            self.config, self.kw = config, kw

    g = Good.Config(x=3).build(extra=5)
    assert g.config.x == 3 and g.kw == {"extra": 5}
    with pytest.raises(ValueError):
        Good.Config().build(x=2)


def test_split_module_and_config():
    m, c, rest = split_module_and_config(["--module=llama3", "--config", "llama3_8b", "--training.steps", "5"])
    assert (m, c, rest) == ("llama3", "llama3_8b", ["--training.steps", "5"])


def test_config_manager_overrides():
    cfg = ConfigManager().parse_args(["--module", "llama3", "--config", "llama3_debugmodel",
                                      "--training.steps", "7", "--optimizer.lr", "0.01"])
    assert cfg.training.steps == 7 and cfg.optimizer.lr == 0.01
    assert cfg.model_spec.flavor == "debugmodel"
    d = cfg.to_dict()
    assert d["model_spec"] == {"name": "llama3", "flavor": "debugmodel"}


def test_kimi_registry_flavors():
    from torchtitan_b200.models.kimi_linear import config_registry as r
    from torchtitan_b200.models.kimi_linear import kimi_linear_args

    for name in ("kimi_linear_194m_baseline", "kimi_linear_48b_block_attn_res", "kimi_linear_528m_full_attn_res"):
        assert callable(getattr(r, name))
    a = kimi_linear_args["48b_baseline"]
    assert a.full_attn_layers == [4, 8, 12, 16, 20, 24, 27] and len(a.kda_layers) == 20
    assert a.num_experts == 256 and a.hidden_size == 2304


def test_parallel_dims():
    class P:
        data_parallel_replicate_degree = 1
        data_parallel_shard_degree = -1
        context_parallel_degree = 2
        tensor_parallel_degree = 2
        pipeline_parallel_degree = 1
        expert_parallel_degree = 4
        expert_tensor_parallel_degree = 1

    pd = ParallelDims.from_config(P, 8)
    assert pd.dp_shard == 2 and pd.fsdp_enabled and pd.seq_len_divisor == 8 and pd.efsdp == 2
    with pytest.raises(ValueError):
        P.pipeline_parallel_degree = 3
        ParallelDims.from_config(P, 8)


def test_wsd_schedule():
    f = lambda s: wsd_factor(s, warmup=2, stable=5, decay=4, kind="linear", min_factor=0.1)  # noqa: E731
    assert f(0) == 0.5 and f(1) == 1.0 and f(3) == 1.0
    assert math.isclose(f(10), 0.1)
    c = wsd_factor(9, warmup=2, stable=5, decay=4, kind="cosine", min_factor=0.0)
    assert 0.0 <= c <= 1.0


def test_synthetic_loader_resume():
    cfg = SyntheticDataLoader.Config(vocab_size=100, pin_memory=False)
    a = cfg.build(dp_rank=1, dp_world_size=2, seq_len=16, local_batch_size=2)
    it = iter(a)
    next(it)
    st = a.state_dict()
    x2, y2 = next(it)
    b = cfg.build(dp_rank=1, dp_world_size=2, seq_len=16, local_batch_size=2)
    b.load_state_dict(st)
    xb, yb = next(iter(b))
    assert torch.equal(x2["input"], xb["input"]) and torch.equal(y2, yb)
    assert torch.equal(x2["input"][:, 1:], y2[:, :-1])
    assert int(x2["input"].max()) < 100


def test_pipeline_fqn_split():
    parts = generate_llm_fqn_per_model_part(4, 6)
    flat = [n for p in parts for n in p]
    assert flat[0] == "tok_embeddings" and flat[-2:] == ["norm", "output"]
    assert [n for n in flat if n.startswith("layers")] == [f"layers.{i}" for i in range(6)]
    assert len(parts) == 4


def test_muon_newton_schulz_orthogonalizes():
    from torchtitan_b200.components.optimizer import zeropower_via_newtonschulz5

    torch.manual_seed(0)
    G = torch.randn(64, 32)
    X = zeropower_via_newtonschulz5(G, steps=5)
    s = torch.linalg.svdvals(X)
    assert s.min() > 0.5 and s.max() < 1.5  # quintic NS pushes all singular values near 1


def test_muon_optimizer_steps():
    from torchtitan_b200.components.optimizer import OptimizersContainer

    m = torch.nn.Sequential(torch.nn.Linear(16, 16, bias=False), torch.nn.LayerNorm(16))
    opt = OptimizersContainer.Config(name="Muon", lr=1e-3, muon_lr=0.02,
                                     muon_exclude_patterns=["1\\."]).build(model_parts=[m])
    groups = opt.optimizers[0].param_groups
    assert any(g["use_muon"] for g in groups) and any(not g["use_muon"] for g in groups)
    w0 = m[0].weight.detach().clone()
    m(torch.randn(4, 16)).sum().backward()
    opt.step()
    assert not torch.equal(w0, m[0].weight)


def test_adamw_matches_torch():
    from torchtitan_b200.components.optimizer import AdamW

    torch.manual_seed(0)
    p1 = torch.nn.Parameter(torch.randn(10, 5))
    p2 = torch.nn.Parameter(p1.detach().clone())
    o1 = AdamW([p1], lr=1e-2, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    o2 = torch.optim.AdamW([p2], lr=1e-2, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    for _ in range(3):
        g = torch.randn(10, 5)
        p1.grad, p2.grad = g.clone(), g.clone()
        o1.step()
        o2.step()
    assert torch.allclose(p1, p2, atol=1e-6)


def test_llama_hf_adapter_roundtrip():
    from torchtitan_b200.models.llama3 import llama3_args
    from torchtitan_b200.models.llama3.state_dict_adapter import Llama3StateDictAdapter

    a = llama3_args["debugmodel"]
    ad = Llama3StateDictAdapter(a)
    sd = {"layers.0.attention.wq.weight": torch.randn(256, 256), "layers.0.attention.wk.weight": torch.randn(128, 256),
          "layers.3.feed_forward.w1.weight": torch.randn(768, 256), "tok_embeddings.weight": torch.randn(2048, 256)}
    hf = ad.to_hf(sd)
    assert "model.layers.0.self_attn.q_proj.weight" in hf and "model.embed_tokens.weight" in hf
    back = ad.from_hf(hf)
    for k, v in sd.items():
        assert torch.equal(back[k], v)


def test_kimi_hf_adapter_roundtrip():
    from torchtitan_b200.models.kimi_linear.state_dict_adapter import KimiLinearStateDictAdapter

    ad = KimiLinearStateDictAdapter()
    sd = {"layers.1.ffn._moe.experts.w1": torch.randn(4, 8, 6), "layers.0.self_attn.A_log": torch.randn(2),
          "layers.1.ffn._moe.router.gate.weight": torch.randn(4, 6), "lm_head.weight": torch.randn(10, 6)}
    hf = ad.to_hf(sd)
    assert "model.layers.1.block_sparse_moe.experts.3.w1.weight" in hf
    back = ad.from_hf(hf)
    for k, v in sd.items():
        assert torch.equal(back[k], v)


def test_moe_forward_backward_and_aux():
    from torchtitan_b200.models.common.moe import MoE

    torch.manual_seed(0)
    m = MoE(16, 32, num_experts=4, top_k=2, route_norm=True, route_scale=2.0, shared_hidden_dim=32,
            aux_loss_coeff=0.01)
    m.init_weights(0.02)
    x = torch.randn(2, 5, 16, requires_grad=True)
    y = m(x)
    y.sum().backward()
    assert y.shape == x.shape and x.grad is not None
    assert m.router.gate.weight.grad is not None and m.last_aux_loss is not None
    assert float(m.tokens_per_expert.sum()) == 2 * 5 * 2


def test_kimi_flops_counts_active_experts_only():
    from torchtitan_b200.models.kimi_linear import build_args

    a = build_args("debugmodel")
    with torch.device("meta"):
        model = a.build()
    n, flops = a.get_nparams_and_flops(model, 128)
    routed = sum(p.numel() for k, p in model.named_parameters() if "_moe.experts." in k)
    assert flops < 6 * (n - routed * 0.5)


def test_fused_clip_matches_explicit_clip():
    from torchtitan_b200.components.optimizer import AdamW
    from torchtitan_b200.parallel.utils import clip_grad_norm_

    torch.manual_seed(1)
    w = torch.randn(6, 4)
    g = torch.randn(6, 4) * 10
    p1, p2 = torch.nn.Parameter(w.clone()), torch.nn.Parameter(w.clone())
    p1.grad, p2.grad = g.clone(), g.clone()
    o1, o2 = AdamW([p1], lr=1e-2), AdamW([p2], lr=1e-2)
    clip_grad_norm_([p1], 1.0)
    o1.step()
    n, total = clip_grad_norm_([p2], 1.0, defer_scaling=True)
    o2.pending_clip = (total, 1.0)
    o2.step()
    assert torch.allclose(p1, p2, atol=1e-6) and o2.pending_clip is None


def test_optimizer_step_in_backward_matches_regular_step(tmp_path):
    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.trainer import Trainer

    def run(extra):
        cfg = ConfigManager().parse_args(["--module", "llama3", "--config", "llama3_debugmodel", "--training.steps",
                                          "3", "--training.seq-len", "128", "--training.local-batch-size", "2",
                                          "--training.dtype", "float32", "--training.mixed-precision-param",
                                          "float32", "--training.max-norm", "0", "--activation-checkpoint.mode",
                                          "none", "--dump-folder", str(tmp_path), *extra])
        torch.manual_seed(0)
        t = Trainer(cfg)
        t.train()
        w = {n: p.detach().clone() for n, p in t.model_parts[0].named_parameters()}
        t.close()
        return w

    a = run([])
    b = run(["--optimizer.early-step-in-backward"])
    for n in a:
        torch.testing.assert_close(a[n], b[n], rtol=1e-5, atol=1e-6)


def test_mx_quantize_rceil_blocks():
    from torchtitan_b200.ops.quant import mx_dequantize, mx_quantize

    torch.manual_seed(0)
    x = torch.randn(4, 64) * torch.logspace(-3, 3, 64)
    q, s = mx_quantize(x)
    assert q.dtype == torch.float8_e4m3fn and s.shape == (4, 2)
    amax = x.view(4, 2, 32).abs().amax(-1)
    exp = s.float() - 127
    assert torch.all(amax / torch.exp2(exp) <= 448) and torch.all(amax / torch.exp2(exp - 1) > 448)
    back = mx_dequantize(q, s, torch.float32)
    rel = ((back - x).abs() / x.view(4, 2, 32).abs().amax(-1).repeat_interleave(32, 1)).max()
    assert rel < 2 ** -3  # e4m3 has 3 mantissa bits


@pytest.mark.parametrize("names", [["mxfp8"], ["float8"], ["float8_rowwise"], ["float8_rowwise_with_gw_hp"]])
def test_quantized_training_converters(names, tmp_path):
    from torchtitan_b200.components.quantization.float8 import Float8Linear
    from torchtitan_b200.components.quantization.mx import MXFP8Linear
    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.trainer import Trainer

    cfg = ConfigManager().parse_args(["--module", "llama3", "--config", "llama3_debugmodel", "--training.steps", "3",
                                      "--training.seq-len", "128", "--training.local-batch-size", "2",
                                      "--training.dtype", "float32", "--training.mixed-precision-param", "float32",
                                      "--activation-checkpoint.mode", "none", "--dump-folder", str(tmp_path),
                                      "--model-converters.names", *names])
    t = Trainer(cfg)
    cls = MXFP8Linear if names == ["mxfp8"] else Float8Linear
    lins = [m for m in t.model_parts[0].modules() if isinstance(m, cls)]
    assert len(lins) == 6 * 7 and type(t.model_parts[0].output) is not cls  # output head excluded
    t.train()
    loss = t.metrics_processor.last_metrics["loss_metrics/global_avg_loss"]
    assert 6.0 < loss < 9.0
    t.close()


def test_mx_linear_gradients_close_to_bf16():
    from torchtitan_b200.components.quantization.mx import _MXLinearFn

    torch.manual_seed(0)
    x = torch.randn(64, 128, requires_grad=True)
    w = torch.randn(96, 128, requires_grad=True)
    y = _MXLinearFn.apply(x, w)
    y.square().sum().backward()
    x2, w2 = x.detach().requires_grad_(), w.detach().requires_grad_()
    (x2 @ w2.t()).square().sum().backward()
    for a, b in ((y, x2 @ w2.t()), (x.grad, x2.grad), (w.grad, w2.grad)):
        assert ((a - b).norm() / b.norm()) < 0.08


def test_chat_dataloader_masks_prompts_and_packs(tmp_path):
    import json

    from torchtitan_b200.components.dataloader import ChatDataLoader
    from torchtitan_b200.components.loss import IGNORE_INDEX

    class CharTok:
        bos_id, eos_id = 1, 2

        def encode(self, text):
            return [3 + (ord(c) % 50) for c in text]

    recs = [{"messages": [{"role": "user", "content": "hi"}, {"role": "assistant", "content": "yo"}]},
            {"messages": [{"role": "user", "content": "abc"}, {"role": "assistant", "content": "de"}]}]
    path = tmp_path / "chat.jsonl"
    path.write_text("\n".join(json.dumps(r) for r in recs))
    dl = ChatDataLoader(ChatDataLoader.Config(dataset_path=str(path), infinite=False), tokenizer=CharTok(),
                        seq_len=64, local_batch_size=1)
    (inp, labels), = list(dl)
    ids, lab, pos = inp["input"][0], labels[0], inp["positions"][0]
    tok = CharTok()
    user1 = tok.encode("<|user|>\nhi\n")
    asst1 = tok.encode("<|assistant|>\nyo\n")
    n1 = 1 + len(user1) + len(asst1) + 1
    # labels are the next tokens; prompt tokens and the leading BOS are ignored
    assert (lab[:len(user1)] == IGNORE_INDEX).all()
    assert lab[len(user1):len(user1) + len(asst1)].tolist() == asst1
    assert lab[len(user1) + len(asst1)] == 2  # eos is trained
    # second sample packed right after the first, positions restart
    assert pos[n1] == 0 and ids[n1] == 1
    assert pos[n1 - 1] == n1 - 1
    n2 = 1 + len(tok.encode("<|user|>\nabc\n")) + len(tok.encode("<|assistant|>\nde\n")) + 1
    assert (lab[n1 + n2 - 1:] == IGNORE_INDEX).all()  # padding


def test_module_protocol_recursive_init():
    import torch.nn as nn

    from torchtitan_b200.protocols.module import Module

    class Block(Module):
        def __init__(self):
            super().__init__()
            self.w = nn.Parameter(torch.empty(4))
            self.lin = Module.from_nn_module(nn.Linear(3, 3), {"weight": nn.init.ones_, "bias": nn.init.zeros_})
            self.plain = nn.Linear(2, 2)
            self.param_init = {"w": lambda t: t.fill_(2.0)}
            self.touched = False

        def init_self(self, buffer_device=None):
            self.touched = True

    b = Block()
    b.plain.weight.data.fill_(123.0)
    b.init_states()
    assert torch.equal(b.w, torch.full((4,), 2.0)) and b.touched
    assert torch.equal(b.lin.weight, torch.ones(3, 3)) and torch.equal(b.lin.bias, torch.zeros(3))
    assert isinstance(b.lin, nn.Linear) and isinstance(b.lin, Module)
    assert not torch.all(b.plain.weight == 123.0)  # reset_parameters ran
    bad = Module.from_nn_module(nn.Linear(2, 2), {"nope": nn.init.zeros_})
    with pytest.raises(KeyError):
        bad.init_states()


def test_quantized_grouped_experts_train(tmp_path):
    from torchtitan_b200.components.quantization.grouped import QuantGroupedExperts
    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.trainer import Trainer

    cfg = ConfigManager().parse_args(["--module", "qwen3", "--config", "qwen3_debugmodel_moe", "--training.steps", "2",
                                      "--training.seq-len", "128", "--training.local-batch-size", "2",
                                      "--training.dtype", "float32", "--training.mixed-precision-param", "float32",
                                      "--activation-checkpoint.mode", "none", "--dump-folder", str(tmp_path),
                                      "--model-converters.names", "mxfp8", "mxfp8_grouped"])
    t = Trainer(cfg)
    assert sum(isinstance(m, QuantGroupedExperts) for m in t.model_parts[0].modules()) == 8
    t.train()
    assert 6.0 < t.metrics_processor.last_metrics["loss_metrics/global_avg_loss"] < 9.0
    t.close()


def test_batch_invariant_env(monkeypatch):
    import os

    from torchtitan_b200.parallel.utils import apply_batch_invariant_env

    for k in ("NCCL_ALGO", "NCCL_PROTO", "NCCL_MIN_NCHANNELS", "NCCL_MAX_NCHANNELS", "NCCL_NVLS_ENABLE",
              "NCCL_COLLNET_ENABLE"):
        monkeypatch.delenv(k, raising=False)
    env = apply_batch_invariant_env()
    assert os.environ["NCCL_ALGO"] == "Ring" and os.environ["NCCL_NVLS_ENABLE"] == "0" and len(env) == 6


def test_grouped_swiglu_padded_reference_matches_loop():
    from torchtitan_b200.ops.grouped import expert_segments, grouped_swiglu_padded

    torch.manual_seed(0)
    counts = torch.tensor([5, 0, 3])
    w1, w3 = torch.randn(3, 6, 4), torch.randn(3, 6, 4)
    w2 = torch.randn(3, 4, 6)
    x = torch.randn(8, 4)
    tg, kst, kln, P = expert_segments(counts)
    assert P == 256 and kst.tolist() == [0, 128, 128]
    xp = torch.zeros(P, 4)
    xp[:5], xp[128:131] = x[:5], x[5:]
    yp = grouped_swiglu_padded(xp, w1, w2, w3, counts)
    f = lambda xs, e: (torch.nn.functional.silu(xs @ w1[e].t()) * (xs @ w3[e].t())) @ w2[e].t()  # noqa: E731
    torch.testing.assert_close(yp[:5], f(x[:5], 0))
    torch.testing.assert_close(yp[128:131], f(x[5:], 2))
    assert torch.count_nonzero(yp[5:128]) == 0


def test_multimodal_dataloader_packs_images(tmp_path):
    import json

    from PIL import Image

    from torchtitan_b200.components.loss import IGNORE_INDEX
    from torchtitan_b200.components.mm_dataloader import MultimodalDataLoader

    for n in ("a.png", "b.png"):
        Image.new("RGB", (40, 30), (255, 0, 0) if n == "a.png" else (0, 0, 255)).save(tmp_path / n)
    recs = [{"text": "see <image> here", "images": ["a.png"]},
            {"text": "two <image> and <image>.", "images": ["a.png", "b.png"]}]
    (tmp_path / "d.jsonl").write_text("\n".join(json.dumps(r) for r in recs))

    class Tok:
        bos_id, eos_id = 1, 2

        def encode(self, t):
            return [3 + ord(ch) % 40 for ch in t]

    dl = MultimodalDataLoader(MultimodalDataLoader.Config(dataset_path=str(tmp_path / "d.jsonl"), image_size=28,
                                                          patch_size=14, infinite=False),
                              tokenizer=Tok(), seq_len=128, local_batch_size=1)
    (inp, labels), = list(dl)
    ids = inp["input"][0]
    assert inp["pixel_values"].shape == (3, 3, 28, 28)
    assert int((ids == -200).sum()) == 12  # 3 images x 4 patches
    full_next = torch.cat([ids[1:], labels[0][-1:]])
    assert (labels[0][full_next == -200] == IGNORE_INDEX).all()
    # red image first, blue last (order of appearance), normalised to [-1, 1]
    assert inp["pixel_values"][0, 0].mean() > 0.9 and inp["pixel_values"][2, 2].mean() > 0.9


def test_peer_watchdog_reports_device_error_word():
    import time

    from torchtitan_b200.parallel.watchdog import ErrorWatchdog, describe

    sink = torch.zeros(8, dtype=torch.int32)
    seen = []
    wd = ErrorWatchdog(sink, interval_s=0.01, on_error=seen.append)
    time.sleep(0.05)
    assert wd.error is None
    sink[1:5] = torch.tensor([3, 17, 2, 16], dtype=torch.int32)
    sink[0] = 71  # written last by the kernel
    for _ in range(200):
        if seen:
            break
        time.sleep(0.01)
    assert seen and seen[0][:5] == [71, 3, 17, 2, 16]
    assert "reduce-scatter wait timed out: slot 3, waiting for epoch 17 from rank 2" in describe(wd.error)
    wd.stop()


def test_mx_blocked_scale_layout_round_trip():
    from torchtitan_b200.ops.mx_gemm import mx_dequantize_ref, mx_gemm, mx_quantize_ref, sf_byte_index
    from torchtitan_b200.ops.quant import mx_fake_quant

    idx = sf_byte_index(130, 256)
    assert idx.shape == (256, 8) and idx.unique().numel() == idx.numel() and int(idx.max()) == 2 * 2 * 512 - 1
    # row 33, group 5 -> record (0, 1), byte 1*16 + 1*4 + 1
    assert int(idx[33, 5]) == 512 + 16 + 4 + 1
    torch.manual_seed(0)
    x = torch.randn(130, 200) * torch.logspace(-2, 2, 200)
    codes, sf = mx_quantize_ref(x)
    assert codes.shape == (130, 256) and sf.numel() == 256 * 256 // 32
    back = mx_dequantize_ref(codes, sf)
    torch.testing.assert_close(back[:, :200], mx_fake_quant(torch.cat([x, torch.zeros(130, 56)], 1), -1)[:, :200],
                               rtol=0, atol=0)
    assert torch.count_nonzero(back[:, 200:]) == 0
    w = torch.randn(70, 200)
    qw, sw = mx_quantize_ref(w)
    y = mx_gemm(codes, sf, qw, sw).float()
    ref = mx_dequantize_ref(codes, sf) @ mx_dequantize_ref(qw, sw).t()
    torch.testing.assert_close(y, ref.bfloat16().float())
    assert ((y - x @ w.t()).norm() / (x @ w.t()).norm()) < 0.08


def test_document_attention_matches_block_causal_mask():
    from torchtitan_b200 import ops
    from torchtitan_b200.models.common.attention import document_causal_mask

    torch.manual_seed(0)
    doc = torch.tensor([[0] * 3 + [1] * 9 + [2] * 4, [0] * 16])
    q, k, v = torch.randn(2, 16, 4, 8), torch.randn(2, 16, 2, 8), torch.randn(2, 16, 2, 8)
    o = ops.document_attention(q, k, v, doc)
    ref = torch.nn.functional.scaled_dot_product_attention(
        q.transpose(1, 2), k.repeat_interleave(2, 2).transpose(1, 2), v.repeat_interleave(2, 2).transpose(1, 2),
        attn_mask=document_causal_mask(doc)).transpose(1, 2)
    assert torch.allclose(o, ref, atol=1e-5)


def test_patchify_matches_hf_qwen2vl_image_processor_layout():
    """Flat patches in merge-block order: row r of block (bh, bw) and intra (mh, mw) holds
    pixels [(bh*m+mh)*P : +P, (bw*m+mw)*P : +P] of every channel, repeated over T."""
    from torchtitan_b200.components.mm_dataloader import patchify

    img = torch.randn(3, 64, 96)
    P, T, m = 16, 2, 2
    x, grid = patchify(img, P, T, m)
    assert grid == [1, 4, 6] and x.shape == (24, 3 * T * P * P)
    r = 0
    for bh in range(2):
        for bw in range(3):
            for mh in range(m):
                for mw in range(m):
                    y0, x0 = (bh * m + mh) * P, (bw * m + mw) * P
                    want = img[:, y0:y0 + P, x0:x0 + P][:, None].expand(3, T, P, P).reshape(-1)
                    assert torch.equal(x[r], want)
                    r += 1


def test_synthetic_image_text_loader_places_images():
    from torchtitan_b200.components.mm_dataloader import SyntheticImageTextDataLoader
    from torchtitan_b200.components.loss import IGNORE_INDEX

    dl = SyntheticImageTextDataLoader(SyntheticImageTextDataLoader.Config(
        images_per_sample=2, image_size=64, patch_size=16, vision_token_id=2046, vocab_size=2048),
        dp_rank=0, dp_world_size=1, seq_len=64, local_batch_size=2)
    inp, labels = next(iter(dl))
    assert inp["pixel_values"].shape == (4 * 16, 3 * 2 * 16 * 16) and inp["grid_thw"].tolist() == [[1, 4, 4]] * 4
    assert int((inp["input"] == 2046).sum()) == 2 * 2 * 4
    assert bool((labels[:, :-1][inp["input"][:, 1:] == 2046] == IGNORE_INDEX).all())
    assert not bool((labels == 2046).any())


def test_peer_dp_launches_buckets_in_index_order():
    """Reduce-scatter kernels wait on the peers' kernels for the same bucket: every rank must
    queue them in the same order, whatever order its gradients arrive in."""
    from types import SimpleNamespace

    from torchtitan_b200.parallel.peer_dp import PeerDataParallel

    dp = PeerDataParallel.__new__(PeerDataParallel)
    dp.buckets = [SimpleNamespace(pending=1, launched=False, index=i) for i in range(4)]
    dp._next_launch = 0
    order = []
    dp._launch = lambda b: order.append(b.index)
    for k in (2, 3, 0, 1):  # gradients complete out of order
        dp.buckets[k].pending = 0
        dp._launch_ready()
        if k == 2:
            assert order == []
    assert order == [0, 1, 2, 3]


def test_compile_flag_falls_back_cleanly_without_cuda(tmp_path):
    """``--compile.enable`` asks for CUDA-graph capture; where it cannot apply (no GPU) the
    trainer says why and trains uncaptured."""
    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.parallel.cuda_graphs import cuda_graphs_applicable
    from torchtitan_b200.trainer import Trainer

    t = Trainer(ConfigManager().parse_args([
        "--module", "llama3", "--config", "llama3_debugmodel_cpu", "--training.steps", "1", "--compile.enable",
        "--training.seq-len", "64", "--dump-folder", str(tmp_path)]))
    assert cuda_graphs_applicable(t.parallel_dims, t.model_parts[0]) is not None
    t.train()
    assert t.step == 1
    t.close()


def test_bitwise_determinism_hashes(tmp_path):
    """Two identically seeded debug runs end with bitwise-identical weights and optimizer
    states; another seed does not (the hashes see every bit)."""
    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.trainer import Trainer
    from torchtitan_b200.utils.hashing import hash_model, hash_optimizer, hash_tensors

    def run(seed):
        t = Trainer(ConfigManager().parse_args([
            "--module", "llama3", "--config", "llama3_debugmodel_cpu", "--training.steps", "2",
            "--training.seq-len", "64", "--debug.seed", str(seed), "--debug.deterministic",
            "--dump-folder", str(tmp_path / str(seed))]))
        t.train()
        out = hash_model(t.model_parts[0]), hash_optimizer(t.optimizers.optimizers[0])
        t.close()
        return out

    a, b, c = run(1), run(1), run(2)
    assert a == b and a[0] != c[0]
    x = torch.zeros(4, dtype=torch.bfloat16)
    y = x.clone()
    y.view(torch.int16)[2] = 1  # one bit
    assert hash_tensors([("w", x)]) != hash_tensors([("w", y)])


def test_huggingface_tokenizer_files(tmp_path):
    """tokenizer.json + tokenizer_config.json: special tokens, round trip, chat template."""
    import json

    from tokenizers import Tokenizer, models, pre_tokenizers

    from torchtitan_b200.components.tokenizer import HuggingFaceTokenizer

    vocab = {w: i for i, w in enumerate(["<unk>", "<s>", "</s>", "hello", "world", "user", "assistant", "hi"])}
    tok = Tokenizer(models.WordLevel(vocab, unk_token="<unk>"))
    tok.pre_tokenizer = pre_tokenizers.Whitespace()
    tok.add_special_tokens(["<s>", "</s>"])
    tok.save(str(tmp_path / "tokenizer.json"))
    (tmp_path / "tokenizer_config.json").write_text(json.dumps({
        "bos_token": "<s>", "eos_token": {"content": "</s>"},
        "chat_template": "{{ bos_token }}{% for m in messages %}{{ m['role'] }} {{ m['content'] }} {% endfor %}"}))
    t = HuggingFaceTokenizer(tokenizer_path=str(tmp_path))
    assert (t.bos_id, t.eos_id) == (1, 2) and t.get_vocab_size() == 8
    ids = t.encode("hello world", add_bos=True, add_eos=True)
    assert ids == [1, 3, 4, 2] and t.decode(ids[1:3]) == "hello world"
    chat = t.apply_chat_template([{"role": "user", "content": "hi"}, {"role": "assistant", "content": "hello"}])
    assert chat == [1, 5, 7, 6, 3]


def test_attnres_stage_cache_sends_only_missing_blocks():
    """Round-robin stages of an AttnRes model: stage s receives only the blocks completed after
    its rank's previous stage (s - pp), plus the partial block."""
    import torch.nn as nn

    from torchtitan_b200.models.common.attn_res import _held, completed_blocks, setup_stage_cache, stage_exit

    assert [completed_blocks(n, 2) for n in range(6)] == [0, 1, 1, 2, 2, 3]
    fqns = [["tok_embeddings", "layers.0"], ["layers.1", "layers.2"], ["layers.3", "layers.4"],
            ["layers.5", "norm", "output"]]
    parts = [nn.Module(), nn.Module()]
    setup_stage_cache(parts, [0, 2], fqns, pp=2, n_microbatches=2, layers_per_block=2)
    cfg = parts[0]._attnres_pp
    assert cfg["counts"] == [1, 2, 3, 3]
    assert [_held(cfg, s) for s in range(4)] == [0, 0, 1, 2]
    # stage 2 (holding 1 block from stage 0) hands stage 3 (holding 2) one block + the partial
    parts[1]._attnres_pp["mb"] = 0
    blocks = [torch.randn(1, 4, 8) for _ in range(3)]
    out = stage_exit(parts[1], (blocks, torch.randn(1, 4, 8)))
    assert out.shape[0] == 2 and torch.equal(out[0], blocks[2])


def test_nonfinite_canary_names_the_module(tmp_path):
    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.trainer import Trainer

    t = Trainer(ConfigManager().parse_args([
        "--module", "llama3", "--config", "llama3_debugmodel_cpu", "--training.steps", "1", "--training.seq-len", "64",
        "--debug.nonfinite-check", "--activation-checkpoint.mode", "none", "--dump-folder", str(tmp_path)]))
    t.train()  # finite: no error
    with torch.no_grad():
        t.model_parts[0].layers["2"].attention.wv.weight.fill_(float("nan"))
    with pytest.raises(FloatingPointError, match=r"layers\.2\.attention\.wv"):
        t.model_parts[0](torch.randint(0, 2048, (1, 16)))
    t.close()
