"""Rollout record passed between the RL actors.

Interface parity: ``experiments/rl/types.py`` (``Episode`` with the same field names, so
graders and controllers written against the reference read these unchanged).
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass
class Episode:
    policy_version: int
    """Weight version of the generator that sampled this completion."""
    prompt_token_ids: list[int]
    text: str
    token_ids: list[int]
    """Completion tokens (the prompt is not repeated here)."""
    token_log_probs: list[float]
    """Generator log-probability of each completion token under the sampling policy."""
    expected_answer: str = ""
    reward: float = 0.0
    group_id: str = ""
    """Completions of one prompt share it; advantages are normalised within a group."""
    advantage: float = 0.0
    image_path: str | None = None


def assign_group_advantages(episodes: list[Episode], normalize_std: bool = False, eps: float = 1e-6) -> None:
    """GRPO advantage: reward minus the group mean (optionally divided by the group std)."""
    groups: dict[str, list[Episode]] = {}
    for e in episodes:
        groups.setdefault(e.group_id, []).append(e)
    for g in groups.values():
        mean = sum(e.reward for e in g) / len(g)
        std = (sum((e.reward - mean) ** 2 for e in g) / len(g)) ** 0.5
        for e in g:
            e.advantage = (e.reward - mean) / (std + eps) if normalize_std else e.reward - mean
