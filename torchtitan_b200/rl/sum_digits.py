"""Sum-of-digits task for the RL example (behaviour parity: ``experiments/rl/sum_digits.py``:
questions over 2-4 integers in [10, 99], answers parsed from an ``[ANSWER] n`` tag, a
natural-language "answer is n", or the last number; reward 1 for a correct answer)."""
from __future__ import annotations

import random
import re

import torch

SYSTEM_PROMPT = ("You are a helpful assistant. Add up every digit of the numbers you are given, "
                 "showing the digits, and finish with [ANSWER] <number>.")


def extract_answer(text: str) -> int | None:
    for pat in (r"\[ANSWER\]\s*(-?\d+)", r"answer(?: is|:)\s*(-?\d+)"):
        found = re.findall(pat, text, flags=re.IGNORECASE)
        if found:
            return int(found[-1])
    nums = re.findall(r"-?\d+", text)
    return int(nums[-1]) if nums else None


class SumDigitsTask:
    def __init__(self, seed: int = 42):
        self.rng = random.Random(seed)

    def create_question(self) -> tuple[str, str]:
        nums = [self.rng.randint(10, 99) for _ in range(self.rng.randint(2, 4))]
        return f"What is the total digit sum of {nums}?", str(sum(int(d) for n in nums for d in str(n)))

    def get_system_prompt(self) -> str:
        return SYSTEM_PROMPT

    @staticmethod
    def reward_function(completions: list[str], expected_answer: str = "") -> torch.Tensor:
        want = int(expected_answer) if expected_answer.lstrip("-").isdigit() else None
        return torch.tensor([1.0 if want is not None and extract_answer(c) == want else 0.0 for c in completions])
