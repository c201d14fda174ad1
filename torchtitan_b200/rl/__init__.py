"""Reinforcement learning on top of the trainer: GRPO in one process (``grpo``) and as
generator / grader / trainer actors with an eager or vLLM generator (``simple_grpo``)."""
from .grpo import GRPOConfig, GRPOTrainer, grpo_loss, group_advantages
from .types import Episode, assign_group_advantages

__all__ = ["GRPOConfig", "GRPOTrainer", "grpo_loss", "group_advantages", "Episode", "assign_group_advantages"]
