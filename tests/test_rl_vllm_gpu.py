"""vLLM generator on a B200: rollouts from an engine built from this framework's weights, their
log-probabilities against this framework's model, and a weight push changing both alike."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ours(margs, state):
    with torch.device("cuda"):
        m = margs.build()
    m.load_state_dict(state, strict=False)
    for p in m.parameters():  # bf16 weights; the RoPE tables (buffers) stay fp32
        p.data = p.data.to(torch.bfloat16)
    return m.eval()


def _logprobs(model, eps):
    from torchtitan_b200.rl.policy_trainer import pack_episodes, sequence_logprobs

    tok, mask, old, _ = pack_episodes(eps, 0, "cuda")
    with torch.no_grad():
        lp = sequence_logprobs(model, tok)
    return lp[mask], old[mask]


def test_vllm_generator_matches_model_and_follows_weight_pushes(tmp_path):
    pytest.importorskip("vllm")
    from torchtitan_b200.models.llama3 import Llama3ModelArgs
    from torchtitan_b200.rl.generators import VLLMGenerator, state_dict_adapter

    torch.manual_seed(0)
    margs = Llama3ModelArgs(dim=512, n_layers=2, n_heads=4, n_kv_heads=2, vocab_size=2048, max_seq_len=512)
    ref = margs.build()
    ref.init_weights()
    state = {k: v.detach().clone() for k, v in ref.state_dict().items() if "freqs" not in k}
    gen = VLLMGenerator("llama3", margs, state_dict_adapter("llama3", margs), state, str(tmp_path),
                        gpu_memory_utilization=0.2)
    prompts = [[11, 12, 13, 14, 15], [7, 8, 9]]
    eps = gen.generate(prompts, n=4, max_new_tokens=8, temperature=1.0, group_ids=["a", "b"])
    assert len(eps) == 8 and all(len(e.token_ids) == 8 for e in eps)
    ours, theirs = _logprobs(_ours(margs, state), eps)
    # bf16 engines: per-token log-probabilities agree to a few hundredths
    assert (ours - theirs).abs().mean() < 0.05, (ours - theirs).abs().max()
    # push different weights: the engine's log-probabilities follow them
    new = {k: (v * 1.5 if k == "output.weight" else v) for k, v in state.items()}
    gen.load_state_dict(new, 1)
    eps2 = gen.generate(prompts, n=4, max_new_tokens=8, temperature=1.0)
    assert all(e.policy_version == 1 for e in eps2)
    ours2, theirs2 = _logprobs(_ours(margs, new), eps2)
    assert (ours2 - theirs2).abs().mean() < 0.05
    old_model_on_new, _ = _logprobs(_ours(margs, state), eps2)
    assert (old_model_on_new - theirs2).abs().mean() > 2 * (ours2 - theirs2).abs().mean()
