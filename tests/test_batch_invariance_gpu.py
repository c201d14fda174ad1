"""Batch invariance of the decoder on a B200: a sequence's per-token log-probabilities do not
depend on which other sequences share the batch, nor on padding after it.  GEMMs accumulate
each output element over K in a fixed order whatever M is, attention and RMSNorm work per row,
so rollouts scored in one batch shape and re-scored by the trainer in another agree bitwise
(the property the reference's RL parity tests require of its inference engine)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_logprobs_independent_of_batch_and_padding():
    from torchtitan_b200.models.llama3 import Llama3ModelArgs
    from torchtitan_b200.ops._ext import ext
    from torchtitan_b200.rl.policy_trainer import sequence_logprobs

    ext()
    torch.manual_seed(0)
    args = Llama3ModelArgs(dim=512, n_layers=2, n_heads=4, n_kv_heads=2, vocab_size=4096, max_seq_len=1024)
    with torch.device("cuda"):
        m = args.build()
    m.init_weights(buffer_device=torch.device("cuda"))
    for p in m.parameters():
        p.data = p.data.to(torch.bfloat16)
    seqs = torch.randint(0, 4096, (8, 320), device="cuda")
    with torch.no_grad():
        alone = sequence_logprobs(m, seqs[:2])                      # batch of 2, length 320
        batched = sequence_logprobs(m, seqs)[:2]                    # batch of 8
        padded = torch.cat([seqs, torch.zeros(8, 192, dtype=seqs.dtype, device="cuda")], 1)
        long = sequence_logprobs(m, padded)[:2, :319]               # 192 padding tokens after
    assert torch.equal(alone, batched), (alone - batched).abs().max()
    assert torch.equal(alone, long), (alone - long).abs().max()
