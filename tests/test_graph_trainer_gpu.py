"""Graph trainer on a B200: the traced step (sm_100a kernels as custom-op nodes) against the
eager step on the same kernels, with the passes and with CUDA-graph replay."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _setup():
    from torchtitan_b200.models.llama3 import Llama3ModelArgs
    from torchtitan_b200.ops._ext import ext

    ext()
    torch.manual_seed(0)
    args = Llama3ModelArgs(dim=512, n_layers=2, n_heads=4, n_kv_heads=2, vocab_size=4096, max_seq_len=512)
    with torch.device("meta"):
        m = args.build()
    m.to_empty(device="cuda")
    m.init_weights()
    for p in m.parameters():
        p.data = p.data.to(torch.bfloat16)
    tok = torch.randint(0, 4096, (2, 256), device="cuda")
    lab = torch.randint(0, 4096, (2, 256), device="cuda")
    return m, tok, lab


def _loss_fn(pred, labels):
    from torchtitan_b200 import ops

    return ops.cross_entropy_sum(pred.flatten(0, 1), labels.flatten())


@pytest.mark.parametrize("cudagraph", [False, True])
def test_traced_step_matches_eager(cudagraph):
    from torchtitan_b200.graph import passes as P
    from torchtitan_b200.graph.cudagraph import CUDAGraphExecutor
    from torchtitan_b200.graph.tracer import GraphStepRunner, trace_train_step

    m, tok, lab = _setup()
    norm = torch.tensor(float(lab.numel()), device="cuda")
    loss = _loss_fn(m(tok), lab) / norm
    loss.backward()
    want = [p.grad.float().clone() for p in m.parameters()]
    tr = trace_train_step(m, _loss_fn, tok, lab, norm)
    names = {str(n.target) for n in tr.gm.graph.nodes}
    assert any("tt_b200.gemm" in t for t in names) and any("tt_b200.attn_fwd" in t for t in names)
    assert any("tt_b200_graph.attn_bwd" in t for t in names) and any("rmsnorm_bwd" in t for t in names)
    P.apply_passes(tr, P.DEFAULT_PASSES + ["selective_recompute"])
    run = GraphStepRunner(m, tr, CUDAGraphExecutor(tr.gm, warmup=1) if cudagraph else None)
    for _ in range(3):  # eager warm-up, capture, replay
        m.zero_grad(set_to_none=True)
        got = run(tok, lab, norm)
        torch.cuda.synchronize()
        torch.testing.assert_close(got.float(), loss.detach().float(), rtol=1e-3, atol=1e-3)
        for p, w in zip(m.parameters(), want):
            torch.testing.assert_close(p.grad.float(), w, rtol=2e-2, atol=2e-3)
    if cudagraph:
        assert run.executor.graph is not None


@pytest.mark.parametrize("family,flavor", [("qwen3", "debugmodel_moe"), ("deepseek_v3", "debugmodel")])
def test_traced_moe_step_matches_eager(family, flavor):
    """MoE debug models (Qwen3-MoE; DeepSeek-V3 with MLA): routing kernel, padded expert layout
    and grouped GEMMs traced as custom-op nodes; the traced step equals the eager step on the
    same kernels."""
    import importlib

    from torchtitan_b200.graph import passes as P
    from torchtitan_b200.graph.tracer import GraphStepRunner, trace_train_step

    spec = importlib.import_module(f"torchtitan_b200.models.{family}").model_registry(flavor)
    torch.manual_seed(0)
    with torch.device("cuda"):
        m = spec.model.build()
    m.init_weights(buffer_device=torch.device("cuda"))
    for p in m.parameters():
        p.data = p.data.to(torch.bfloat16)
    V = spec.model.vocab_size
    tok = torch.randint(0, V, (2, 256), device="cuda")
    lab = torch.randint(0, V, (2, 256), device="cuda")
    norm = torch.tensor(float(lab.numel()), device="cuda")
    loss = _loss_fn(m(tok), lab) / norm
    loss.backward()
    want = [p.grad.float().clone() for p in m.parameters()]
    m.zero_grad(set_to_none=True)
    tr = trace_train_step(m, _loss_fn, tok, lab, norm)
    names = {str(n.target) for n in tr.gm.graph.nodes}
    assert any("gemm_grouped_rows" in t for t in names) and any("router_topk" in t for t in names)
    P.apply_passes(tr, P.DEFAULT_PASSES)
    got = GraphStepRunner(m, tr)(tok, lab, norm)
    torch.cuda.synchronize()
    torch.testing.assert_close(got.float(), loss.detach().float(), rtol=1e-3, atol=1e-3)
    for p, w in zip(m.parameters(), want):
        torch.testing.assert_close(p.grad.float(), w, rtol=2e-2, atol=2e-3)
