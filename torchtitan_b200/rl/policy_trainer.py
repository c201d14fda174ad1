"""Policy trainer of the RL loop: consumes scored episodes, takes one optimizer step on the
clipped GRPO surrogate, and hands its weights to the generator.

Role parity: ``experiments/rl/actors/trainer.py`` (``PolicyTrainer.step(episodes)``,
``push_model_state_dict``) and ``actors/utils.py`` (``compute_token_log_probs``,
``compute_policy_gradient_loss``, ``verify_logprob_identity``).  The update runs through
:class:`~torchtitan_b200.forge.ForgeEngine`, so the trainer's parallelism, optimizer, clipping
and LR schedule apply; the "old" log-probabilities are the generator's, so the importance
ratio measures generator/trainer mismatch as well as policy staleness.
"""
from __future__ import annotations

from typing import Any

import torch

from .grpo import grpo_loss
from .types import Episode


def pack_episodes(episodes: list[Episode], pad_id: int, device) -> tuple[torch.Tensor, ...]:
    """Right-padded token matrix ``[N, T]``, the index of each completion's first token, the
    completion mask over positions ``1..T-1`` (targets), old log-probs and advantages."""
    seqs = [e.prompt_token_ids + e.token_ids for e in episodes]
    T = max(len(s) for s in seqs)
    tok = torch.full((len(seqs), T), pad_id, dtype=torch.long)
    mask = torch.zeros(len(seqs), T - 1, dtype=torch.bool)
    old = torch.zeros(len(seqs), T - 1)
    for i, (e, s) in enumerate(zip(episodes, seqs)):
        tok[i, :len(s)] = torch.tensor(s)
        a, b = len(e.prompt_token_ids) - 1, len(s) - 1  # targets of the completion tokens
        mask[i, a:b] = True
        old[i, a:b] = torch.tensor(e.token_log_probs[: b - a], dtype=torch.float32)
    adv = torch.tensor([e.advantage for e in episodes], dtype=torch.float32)
    return tok.to(device), mask.to(device), old.to(device), adv.to(device)


def sequence_logprobs(model, tok: torch.Tensor) -> torch.Tensor:
    """log p(tok[:, t+1] | tok[:, :t+1]) for every position: ``[N, T-1]``."""
    logits = model(tok[:, :-1]).float()
    return torch.log_softmax(logits, -1).gather(-1, tok[:, 1:, None]).squeeze(-1)


def verify_logprob_identity(episodes: list[Episode], model, pad_id: int = 0, device="cpu") -> float:
    """Largest |trainer log-prob - generator log-prob| over the episodes' completion tokens
    (0 when generator and trainer compute the same numbers)."""
    tok, mask, old, _ = pack_episodes(episodes, pad_id, device)
    with torch.no_grad():
        lp = sequence_logprobs(model, tok)
    return float(((lp - old).abs() * mask).max()) if bool(mask.any()) else 0.0


class PolicyTrainer:
    """Builds a :class:`ForgeEngine` from ``--module/--config`` style arguments."""

    def __init__(self, argv: list[str], clip_eps: float = 0.2, pad_id: int = 0):
        from torchtitan_b200.config.manager import ConfigManager
        from torchtitan_b200.forge import ForgeEngine

        self.engine = ForgeEngine(ConfigManager().parse_args(argv))
        self.clip_eps = clip_eps
        self.pad_id = pad_id
        self.version = 0

    @property
    def device(self):
        return self.engine.trainer.device

    def model_args(self) -> Any:
        return self.engine.trainer.model_args

    def push_model_state_dict(self) -> tuple[dict[str, torch.Tensor], int]:
        """Full (gathered) parameters on the CPU, and their version."""
        out = {}
        for n, p in self.engine.model_parts[0].named_parameters():
            t = p.full_tensor() if hasattr(p, "full_tensor") else p
            out[n] = t.detach().to("cpu", copy=True)
        return out, self.version

    def step(self, episodes: list[Episode]) -> dict[str, float]:
        tok, mask, old, adv = pack_episodes(episodes, self.pad_id, self.device)

        def objective(model):
            lp = sequence_logprobs(model, tok)
            return grpo_loss(lp, old, adv, mask, self.clip_eps)

        loss = float(self.engine.step_with_loss(objective))
        self.version += 1
        rewards = torch.tensor([e.reward for e in episodes])
        return {"loss": loss, "reward_mean": float(rewards.mean()), "version": self.version,
                "n_tokens": int(mask.sum())}

    def logprob_mismatch(self, episodes: list[Episode]) -> float:
        return verify_logprob_identity(episodes, self.engine.model_parts[0], self.pad_id, self.device)

    def close(self) -> None:
        self.engine.close()

