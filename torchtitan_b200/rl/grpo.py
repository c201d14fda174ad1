"""Group Relative Policy Optimisation (behaviour parity: reference
``experiments/rl/simple_grpo_sum_digits.py``; Shao et al. 2024, "DeepSeekMath").

One step:
1. the generator (a copy of the policy, weights synced from the trainer) samples
   ``group_size`` completions per prompt;
2. a reward function scores every completion; advantages are the rewards
   normalised within each prompt's group, ``(r - mean) / (std + eps)``;
3. the policy is updated on the clipped surrogate
   ``-min(rho * A, clip(rho, 1-eps, 1+eps) * A)`` per completion token
   (``rho`` = new / old token probability) plus ``kl_coeff`` times the k3
   estimator of KL(policy || reference), averaged over completion tokens.

Rollouts come from this framework's own model and ``generate`` (the reference
uses vLLM / SGLang actors); the trainer side is ``forge.ForgeEngine``, so every
parallelism of the trainer applies to the update.  Generation runs on the
generator's full copy of the weights in one process.
"""
from __future__ import annotations

import copy
from collections.abc import Callable
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from torchtitan_b200.generate import generate


@dataclass
class GRPOConfig:
    group_size: int = 8
    max_new_tokens: int = 16
    temperature: float = 1.0
    top_k: int = 0
    clip_eps: float = 0.2
    kl_coeff: float = 0.0
    update_epochs: int = 1
    seed: int = 0


def group_advantages(rewards: torch.Tensor, group_size: int, eps: float = 1e-6) -> torch.Tensor:
    r = rewards.view(-1, group_size).float()
    return ((r - r.mean(1, keepdim=True)) / (r.std(1, keepdim=True, unbiased=False) + eps)).view(-1)


def token_logprobs(model, seq: torch.Tensor, start: int) -> torch.Tensor:
    """log p(seq[:, t] | seq[:, :t]) for t >= start: [N, T - start]."""
    logits = model(seq[:, :-1]).float()
    lp = F.log_softmax(logits[:, start - 1:], dim=-1)
    return lp.gather(-1, seq[:, start:, None]).squeeze(-1)


def grpo_loss(lp_new: torch.Tensor, lp_old: torch.Tensor, adv: torch.Tensor, mask: torch.Tensor,
              clip_eps: float, lp_ref: torch.Tensor | None = None, kl_coeff: float = 0.0) -> torch.Tensor:
    ratio = torch.exp(lp_new - lp_old)
    a = adv[:, None]
    surrogate = torch.minimum(ratio * a, ratio.clamp(1 - clip_eps, 1 + clip_eps) * a)
    per_tok = -surrogate
    if lp_ref is not None and kl_coeff > 0:
        d = lp_ref - lp_new
        per_tok = per_tok + kl_coeff * (torch.exp(d) - d - 1)  # k3 estimator, >= 0
    m = mask.float()
    return (per_tok * m).sum() / m.sum().clamp_min(1)


class GRPOTrainer:
    def __init__(self, engine, reward_fn: Callable[[torch.Tensor, torch.Tensor], torch.Tensor],
                 cfg: GRPOConfig | None = None, eos_id: int | None = None):
        self.engine = engine
        self.reward_fn = reward_fn
        self.cfg = cfg or GRPOConfig()
        self.eos_id = eos_id
        # unsharded copies built from the model config (the trainer's model may be
        # FSDP/TP-sharded, which neither deep-copies nor generates token by token)
        self.generator = self._build_copy()
        self.reference = None
        if self.cfg.kl_coeff > 0:
            self.sync_weights()
            self.reference = copy.deepcopy(self.generator)
        self.gen = torch.Generator(device=engine.trainer.device).manual_seed(self.cfg.seed)

    def _build_copy(self):
        t = self.engine.trainer
        with torch.device(t.device):
            m = t.model_args.build()
        m.init_weights()
        for p in m.parameters():
            p.requires_grad_(False)
        return m.eval()

    @torch.no_grad()
    def sync_weights(self) -> None:
        """Trainer -> generator weight sync (full tensors; sharded parameters are gathered)."""
        src = dict(self.engine.model_parts[0].named_parameters())
        for n, p in self.generator.named_parameters():
            s = src[n]
            p.copy_(s.full_tensor() if hasattr(s, "full_tensor") else s)

    def step(self, prompts: torch.Tensor) -> dict[str, float]:
        c = self.cfg
        dev = self.engine.trainer.device
        prompts = prompts.to(dev)
        self.sync_weights()
        P, L = prompts.shape
        rep = prompts.repeat_interleave(c.group_size, 0)
        with torch.no_grad():
            seq = generate(self.generator, rep, c.max_new_tokens, c.temperature, c.top_k, self.gen, self.eos_id)
            completion = seq[:, L:]
            rewards = self.reward_fn(rep, completion).float().to(dev)
            adv = group_advantages(rewards, c.group_size)
            lp_old = token_logprobs(self.generator, seq, L)
            lp_ref = token_logprobs(self.reference, seq, L) if self.reference is not None else None
            mask = torch.ones_like(completion, dtype=torch.bool)
            if self.eos_id is not None:  # tokens after the first EOS are padding
                after = (completion == self.eos_id).int().cumsum(1) - (completion == self.eos_id).int()
                mask = after == 0
        losses = []
        for _ in range(c.update_epochs):
            def loss_fn(model):
                return grpo_loss(token_logprobs(model, seq, L), lp_old, adv, mask, c.clip_eps, lp_ref, c.kl_coeff)

            losses.append(float(self.engine.step_with_loss(loss_fn)))
        return {"reward_mean": float(rewards.mean()), "reward_max": float(rewards.max()), "loss": losses[-1]}
