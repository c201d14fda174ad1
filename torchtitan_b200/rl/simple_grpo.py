"""GRPO with separate generator, grader and trainer actors.

Role parity: ``experiments/rl/simple_grpo_sum_digits.py`` (controller loop over Monarch actors:
weight push -> rollouts -> grading -> group advantages -> policy step).  Here every actor is a
process of :mod:`.actors`; the generator is this framework's decoder (``--generator eager``)
or vLLM (``--generator vllm``, one GPU), the trainer a :class:`~.policy_trainer.PolicyTrainer`.

  python -m torchtitan_b200.rl.simple_grpo --steps 20 --generator eager -- \
      --module qwen3 --config qwen3_debugmodel --hf-assets-path <tokenizer dir>
"""
from __future__ import annotations

import argparse
import asyncio
import re
from typing import Callable

import torch

from torchtitan_b200.utils.logging import init_logger, logger

from .actors import ActorHandle, Provisioner
from .types import Episode, assign_group_advantages


class Grader:
    """Scores each episode with ``reward_fn([text], expected_answer)`` (parity:
    ``experiments/rl/actors/grader.py``)."""

    def __init__(self, reward_fn: Callable):
        self.reward_fn = reward_fn

    def score(self, episodes: list[Episode]) -> list[Episode]:
        for e in episodes:
            e.reward = float(self.reward_fn([e.text], e.expected_answer)[0])
        return episodes


def low_token_reward(completions: list[str], expected_answer: str = "") -> torch.Tensor:
    """Toy reward without a tokenizer: the fraction of completion token ids below 1024
    (completions are the ids joined by spaces)."""
    out = []
    for c in completions:
        ids = [int(x) for x in re.findall(r"\d+", c)]
        out.append(sum(i < 1024 for i in ids) / max(len(ids), 1))
    return torch.tensor(out)


def make_generator(kind: str, model_args, state, gpus, workdir: str,
                   tokenizer_path: str | None, family: str) -> ActorHandle:
    if kind == "eager":
        from .generators import EagerGenerator

        dev = "cuda" if gpus else "cpu"
        return ActorHandle(EagerGenerator, model_args, device=dev, dtype="bfloat16" if gpus else "float32",
                           tokenizer_path=tokenizer_path, gpus=gpus)
    if kind == "vllm":
        from .generators import VLLMGenerator, state_dict_adapter

        adapter = state_dict_adapter(family, model_args)
        return ActorHandle(VLLMGenerator, family, model_args, adapter, state, workdir,
                           tokenizer_path=tokenizer_path, gpus=gpus)
    raise ValueError(f"unknown generator {kind!r}")


async def run(args, trainer_argv: list[str]) -> list[dict]:
    from .policy_trainer import PolicyTrainer

    prov = Provisioner(args.ngpu) if args.ngpu else None
    trainer = ActorHandle(PolicyTrainer, trainer_argv, gpus=prov.allocate(1) if prov else None,
                          env={"MASTER_PORT": str(args.port)})
    try:
        margs = await trainer.model_args()
        state, version = await trainer.push_model_state_dict()
        gen = make_generator(args.generator, margs, state, prov.allocate(1) if prov else None,
                             args.workdir, args.tokenizer, args.family)
        grader = ActorHandle(Grader, low_token_reward)
        g = torch.Generator().manual_seed(args.seed)
        history = []
        try:
            for step in range(args.steps):
                await gen.load_state_dict(state, version)
                prompts = torch.randint(0, margs.vocab_size, (args.prompts, args.prompt_len), generator=g).tolist()
                eps = await gen.generate(prompts, args.group_size, args.max_new_tokens, args.temperature,
                                         group_ids=[f"{step}-{i}" for i in range(len(prompts))])
                eps = await grader.score(eps)
                assign_group_advantages(eps)
                m = await trainer.step(eps)
                m["step"] = step
                history.append(m)
                logger.info(f"rl step {step}: reward {m['reward_mean']:.3f} loss {m['loss']:.4f}")
                state, version = await trainer.push_model_state_dict()
        finally:
            gen.stop()
            grader.stop()
        return history
    finally:
        trainer.stop()


def parse(argv: list[str] | None = None):
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--generator", choices=("eager", "vllm"), default="eager")
    p.add_argument("--family", default="llama3")
    p.add_argument("--ngpu", type=int, default=0, help="0: everything on the CPU")
    p.add_argument("--prompts", type=int, default=4)
    p.add_argument("--prompt-len", type=int, default=8)
    p.add_argument("--group-size", type=int, default=8)
    p.add_argument("--max-new-tokens", type=int, default=8)
    p.add_argument("--temperature", type=float, default=1.0)
    p.add_argument("--tokenizer", default=None)
    p.add_argument("--workdir", default="./outputs/rl")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--port", type=int, default=29531)
    args, rest = p.parse_known_args(argv)
    if rest and rest[0] == "--":
        rest = rest[1:]
    return args, rest


def main(argv: list[str] | None = None) -> list[dict]:
    init_logger()
    args, trainer_argv = parse(argv)
    return asyncio.run(run(args, trainer_argv))


if __name__ == "__main__":
    main()
