"""The Qwen3 / DeepSeek-V3 / Llama 4 / GPT-OSS debug models on a B200: one bf16
forward+backward through the tcgen05 kernels, compared with the same model
run in fp32 PyTorch on the same device."""
import importlib

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("module,flavor", [("qwen3", "debugmodel"), ("qwen3", "debugmodel_moe"),
                                           ("deepseek_v3", "debugmodel"), ("llama4", "debugmodel"),
                                           ("gpt_oss", "debugmodel")])
def test_family_bf16_forward_backward(module, flavor):
    spec = importlib.import_module(f"torchtitan_b200.models.{module}").model_registry(flavor)
    torch.manual_seed(0)
    with torch.device("cuda"):
        model = spec.model.build()
    model.init_weights(buffer_device=torch.device("cuda"))
    for p in model.parameters():
        p.data = p.data.bfloat16()
    tokens = torch.randint(0, spec.model.vocab_size, (1, 512), device="cuda")
    logits = model(tokens)
    loss = F.cross_entropy(logits.flatten(0, 1).float(), tokens.roll(-1, 1).flatten())
    loss.backward()
    assert torch.isfinite(loss) and 6.0 < float(loss) < 10.0
    grads = [p.grad for p in model.parameters()]
    assert all(g is not None and torch.isfinite(g).all() for g in grads)
