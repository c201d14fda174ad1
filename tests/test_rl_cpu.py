"""GRPO (reference ``experiments/rl``): advantage/loss math and a learning run on
the debug model with a toy reward (CPU)."""
import torch

from torchtitan_b200.rl import GRPOConfig, GRPOTrainer, group_advantages, grpo_loss


def test_group_advantages_normalise_within_groups():
    r = torch.tensor([1.0, 0.0, 1.0, 0.0, 5.0, 5.0, 5.0, 5.0])
    a = group_advantages(r, 4)
    assert torch.allclose(a[:4], torch.tensor([1.0, -1.0, 1.0, -1.0]), atol=1e-4)
    assert torch.all(a[4:] == 0)  # a group with one reward carries no signal


def test_grpo_loss_is_reinforce_on_policy_and_kl_vanishes_at_reference():
    torch.manual_seed(0)
    lp = torch.randn(4, 5).requires_grad_()
    adv = torch.randn(4)
    mask = torch.ones(4, 5, dtype=torch.bool)
    mask[0, 3:] = False
    loss = grpo_loss(lp, lp.detach(), adv, mask, 0.2, lp.detach(), kl_coeff=0.5)
    loss.backward()
    # at ratio 1 the clipped surrogate's gradient is -A / n_tokens and k3's gradient is 0
    want = -(adv[:, None] * mask) / mask.sum()
    assert torch.allclose(lp.grad, want, atol=1e-6)
    # clipping: beyond 1 + eps a positive advantage contributes no gradient
    lp2 = (lp.detach() + 1.0).requires_grad_()
    grpo_loss(lp2, lp.detach(), adv.abs(), mask, 0.2).backward()
    assert torch.all(lp2.grad == 0)


def test_grpo_improves_reward(tmp_path):
    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.forge import ForgeEngine

    cfg = ConfigManager().parse_args([
        "--module", "llama3", "--config", "llama3_debugmodel", "--training.seq-len", "64",
        "--training.local-batch-size", "2", "--training.dtype", "float32", "--training.mixed-precision-param",
        "float32", "--activation-checkpoint.mode", "none", "--dump-folder", str(tmp_path), "--optimizer.lr", "3e-3",
        "--lr-scheduler.warmup-steps", "1", "--training.steps", "1000", "--lr-scheduler.decay-ratio", "0.0"])
    eng = ForgeEngine(cfg)

    def reward(prompt, completion):  # fraction of completion tokens in the lower half of the vocabulary
        return (completion < 1024).float().mean(1)

    tr = GRPOTrainer(eng, reward, GRPOConfig(group_size=8, max_new_tokens=8, kl_coeff=0.01, update_epochs=2))
    g = torch.Generator().manual_seed(0)
    hist = [tr.step(torch.randint(0, 2048, (4, 8), generator=g))["reward_mean"] for _ in range(25)]
    assert eng.step == 50
    assert sum(hist[-5:]) / 5 > sum(hist[:5]) / 5 + 0.08, hist
    eng.close()


def test_generator_and_trainer_logprobs_are_bitwise_equal(tmp_path):
    """Rollout log-probabilities (generator copy) and the trainer's own, on the same weights,
    are bitwise equal, so the importance ratio is exactly 1 on the first update epoch
    (the reference checks this parity between its inference engine and trainer)."""
    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.forge import ForgeEngine
    from torchtitan_b200.rl.grpo import token_logprobs

    cfg = ConfigManager().parse_args([
        "--module", "llama3", "--config", "llama3_debugmodel", "--training.seq-len", "64",
        "--training.local-batch-size", "2", "--training.dtype", "float32", "--training.mixed-precision-param",
        "float32", "--activation-checkpoint.mode", "none", "--dump-folder", str(tmp_path)])
    eng = ForgeEngine(cfg)
    tr = GRPOTrainer(eng, lambda p, c: torch.zeros(c.shape[0]), GRPOConfig(group_size=2, max_new_tokens=4))
    tr.sync_weights()
    seq = torch.randint(0, 2048, (4, 12), generator=torch.Generator().manual_seed(0))
    with torch.no_grad():
        a = token_logprobs(tr.generator, seq, 8)
        b = token_logprobs(eng.model_parts[0], seq, 8)
    assert torch.equal(a, b)
    eng.close()
