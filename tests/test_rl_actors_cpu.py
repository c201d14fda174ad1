"""RL actors on CPU: episodes and advantages, the sum-digits task, generator/trainer log-prob
identity, actor error propagation, and the actor GRPO loop end to end."""
import torch

from torchtitan_b200.rl.types import Episode, assign_group_advantages

_TRAINER_ARGS = ["--module", "llama3", "--config", "llama3_debugmodel", "--training.seq-len", "64",
                 "--training.local-batch-size", "2", "--training.dtype", "float32",
                 "--training.mixed-precision-param", "float32", "--activation-checkpoint.mode", "none",
                 "--optimizer.lr", "3e-3", "--lr-scheduler.warmup-steps", "1", "--lr-scheduler.decay-ratio", "0.0"]


def test_group_advantages_are_reward_minus_group_mean():
    eps = [Episode(0, [1], "", [2], [0.0], reward=r, group_id=g)
           for r, g in ((1.0, "a"), (0.0, "a"), (3.0, "b"), (3.0, "b"))]
    assign_group_advantages(eps)
    assert [e.advantage for e in eps] == [0.5, -0.5, 0.0, 0.0]
    assign_group_advantages(eps, normalize_std=True)
    assert abs(eps[0].advantage - 1.0) < 1e-4


def test_sum_digits_task():
    from torchtitan_b200.rl.sum_digits import SumDigitsTask, extract_answer

    assert extract_answer("1 + 2 = 3 [ANSWER] 3") == 3
    assert extract_answer("so the answer is 17.") == 17
    assert extract_answer("first 4 then 9") == 9 and extract_answer("none") is None
    t = SumDigitsTask(seed=1)
    q, a = t.create_question()
    nums = [int(x) for x in q[q.index("[") + 1:q.index("]")].split(",")]
    assert 2 <= len(nums) <= 4 and all(10 <= n <= 99 for n in nums)
    assert int(a) == sum(int(d) for n in nums for d in str(n))
    r = t.reward_function([f"[ANSWER] {a}", "[ANSWER] -1"], a)
    assert r.tolist() == [1.0, 0.0]


def test_generator_logprobs_match_trainer(tmp_path):
    from torchtitan_b200.rl.generators import EagerGenerator
    from torchtitan_b200.rl.policy_trainer import PolicyTrainer

    pt = PolicyTrainer(_TRAINER_ARGS + ["--dump-folder", str(tmp_path)])
    gen = EagerGenerator(pt.model_args())
    state, v = pt.push_model_state_dict()
    gen.load_state_dict(state, v)
    prompts = [[5, 6, 7, 8], [9, 10, 11]]  # two prompt lengths
    eps = gen.generate(prompts, n=3, max_new_tokens=5, group_ids=["x", "y"])
    assert len(eps) == 6 and all(len(e.token_ids) == 5 and len(e.token_log_probs) == 5 for e in eps)
    assert {e.group_id for e in eps} == {"x", "y"}
    # the trainer recomputes exactly the generator's log-probabilities on the same weights
    assert pt.logprob_mismatch(eps) < 1e-5
    for e in eps:
        e.reward = float(len(e.token_ids))
    assign_group_advantages(eps)
    m = pt.step(eps)
    assert m["version"] == 1 and m["n_tokens"] == 30
    # after the update the weights differ, so the generator's old log-probs no longer match
    assert pt.logprob_mismatch(eps) > 1e-6
    pt.close()


class _Boom:
    def __init__(self, x):
        self.x = x

    def ok(self):
        return self.x + 1

    def fail(self):
        raise ValueError("boom")


def test_actor_calls_and_errors():
    import asyncio

    import pytest

    from torchtitan_b200.rl.actors import ActorError, ActorHandle, Provisioner

    a = ActorHandle(_Boom, 41)
    try:
        assert asyncio.run(a.ok()) == 42
        with pytest.raises(ActorError, match="boom"):
            a.call_sync("fail")
        assert a.call_sync("ok") == 42  # the actor survives a failed call
    finally:
        a.stop()
    p = Provisioner(4)
    assert p.allocate(3) == [0, 1, 2]
    with pytest.raises(RuntimeError):
        p.allocate(2)


def test_actor_grpo_loop(tmp_path):
    from torchtitan_b200.rl.simple_grpo import main

    hist = main(["--steps", "3", "--workdir", str(tmp_path), "--port", "29547", "--"] + _TRAINER_ARGS
                + ["--dump-folder", str(tmp_path)])
    assert [h["version"] for h in hist] == [1, 2, 3]
    assert all(0.0 <= h["reward_mean"] <= 1.0 and h["n_tokens"] == 4 * 8 * 8 for h in hist)
