"""Reinforcement learning on top of the trainer (GRPO)."""
from .grpo import GRPOConfig, GRPOTrainer, grpo_loss, group_advantages

__all__ = ["GRPOConfig", "GRPOTrainer", "grpo_loss", "group_advantages"]
