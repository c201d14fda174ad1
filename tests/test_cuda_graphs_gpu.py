"""CUDA-graph capture of decoder blocks (``compile.enable``, backend ``cudagraph``):
a captured Llama debug model gives the same loss and gradients as the uncaptured one."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("family,flavor", [("llama3", "debugmodel"), ("qwen3", "debugmodel_moe")])
def test_graphed_blocks_match_eager(family, flavor):
    """Dense blocks, and MoE blocks (fused routing kernel, padded expert layout: no host read)."""
    import importlib

    from torchtitan_b200.components.loss import cross_entropy_loss
    from torchtitan_b200.parallel.cuda_graphs import apply_cuda_graphs

    spec = importlib.import_module(f"torchtitan_b200.models.{family}").model_registry(flavor)
    V = spec.model.vocab_size
    torch.manual_seed(0)
    with torch.device("cuda"):
        eager = spec.model.build()
        graphed = spec.model.build()
    eager.init_weights(buffer_device=torch.device("cuda"))
    graphed.load_state_dict(eager.state_dict())
    graphed.rope.init_weights(torch.device("cuda"))
    for m in (eager, graphed):
        for p in m.parameters():
            p.data = p.data.bfloat16()
        m.train()
    assert apply_cuda_graphs(graphed, 2, 256, torch.bfloat16) == len(graphed.layers)
    for step in range(3):
        tok = torch.randint(0, V, (2, 257), device="cuda", generator=torch.Generator("cuda").manual_seed(step))
        losses = []
        for m in (eager, graphed):
            m.zero_grad(set_to_none=True)
            loss = cross_entropy_loss(m(tok[:, :-1]), tok[:, 1:]) / tok[:, 1:].numel()
            loss.backward()
            losses.append(float(loss))
        assert abs(losses[0] - losses[1]) < 1e-3 * abs(losses[0])
        for (n, a), b in zip(eager.named_parameters(), graphed.parameters()):
            assert float((a.grad.float() - b.grad.float()).abs().max()) <= 2e-2 * float(a.grad.float().abs().max()) + 1e-6, n
    with torch.no_grad():  # eval / no-grad falls back to the blocks' own forward
        tok = torch.randint(0, V, (1, 100), device="cuda")
        assert torch.allclose(eager(tok).float(), graphed(tok).float(), atol=2e-2, rtol=2e-2)
