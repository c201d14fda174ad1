"""Fault-tolerant replicas on CPU (gloo): each replica is its own process with no shared
default group; they meet at a lighthouse store. A replica that leaves between steps is
dropped from the next quorum after the quorum timeout and the others keep training in
lock-step; a replica that starts late heals from the most advanced one and then matches it."""
import json
import multiprocessing as mp
import os
import tempfile
import time

import pytest
import torch


def _replica(rid, address, group_size, steps, out, stop_after=None, start_delay=0.0, seed=0, wait_for=(),
             step_time=0.0, join_after_round=None):
    import torch.nn as nn

    from torchtitan_b200.parallel.ft import FTManager

    time.sleep(start_delay)
    torch.manual_seed(seed)
    model = nn.Sequential(nn.Linear(16, 32), nn.Tanh(), nn.Linear(32, 4))
    opt = torch.optim.SGD(model.parameters(), lr=0.05, momentum=0.9)
    ft = FTManager(address, rid, group_size, min_replica_size=2, quorum_timeout_s=1.0, collective_timeout_s=5.0)
    # process start-up takes seconds: replicas that should start together wait for each other
    ft.store.set(f"ready/{rid}", "1")
    ft.store.wait([f"ready/{r}" for r in wait_for])
    if join_after_round is not None:  # a late replica: arrive once the others have trained a while
        while not (ft.store.check(["latest"]) and int(ft.store.get("latest").decode()) >= join_after_round):
            time.sleep(0.01)
    my_step, log, commits = 0, [], 0
    while my_step < steps:
        q = ft.start_quorum(my_step)
        if ft.heal([model], opt):
            my_step = q.source_step
            if my_step >= steps:
                break
        g = torch.Generator().manual_seed(1000 * my_step + rid)
        x = torch.randn(8, 16, generator=g)
        y = torch.randn(8, 4, generator=g)
        torch.nn.functional.mse_loss(model(x), y).backward()
        ok = ft.allreduce_gradients([model])
        if ft.should_commit(ok):
            opt.step()
            my_step += 1
            commits += 1
        opt.zero_grad()
        time.sleep(step_time)  # stands in for real step time, so a late replica arrives mid-run
        log.append({"round": q.qid, "participants": q.participants, "step": my_step})
        if os.environ.get("FT_DEBUG"):
            print(rid, q.qid, q.participants, my_step, ok, flush=True)
        if stop_after is not None and commits >= stop_after:
            break
    flat = torch.cat([p.detach().reshape(-1) for p in model.parameters()])
    with open(os.path.join(out, f"r{rid}.json"), "w") as f:
        json.dump({"log": log, "weights": flat.tolist(), "step": my_step}, f)


def _run(specs, group_size, steps):
    from torchtitan_b200.parallel.ft import Lighthouse

    lh = Lighthouse(0)
    ctx = mp.get_context("spawn")
    with tempfile.TemporaryDirectory() as d:
        procs = [ctx.Process(target=_replica, args=(rid, lh.address, group_size, steps, d), kwargs=kw)
                 for rid, kw in specs]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
            assert p.exitcode == 0, f"replica exited with {p.exitcode}"
        return {rid: json.load(open(os.path.join(d, f"r{rid}.json"))) for rid, _ in specs}


def test_replica_loss_leaves_survivors_in_lockstep():
    together = {"wait_for": (0, 1, 2)}
    res = _run([(0, together), (1, together), (2, {"stop_after": 3, **together})], group_size=3, steps=8)
    assert 3 <= res[2]["step"] < 8  # three committed steps (more if it healed forward first)
    for rid in (0, 1):
        parts = [e["participants"] for e in res[rid]["log"]]
        # who makes the first rounds depends on start-up timing; all three train together at
        # some point, and after replica 2 leaves the survivors continue as a pair
        assert [0, 1, 2] in parts and parts[-1] == [0, 1], parts
        assert res[rid]["step"] == 8
    assert res[0]["weights"] == res[1]["weights"]


def test_late_replica_heals_from_peer():
    pair = {"wait_for": (0, 1), "step_time": 0.05}
    res = _run([(0, pair), (1, pair), (2, {"join_after_round": 20, "seed": 7, "step_time": 0.05})], group_size=3,
               steps=200)
    for rid in (0, 1, 2):
        assert res[rid]["step"] == 200, (rid, res[rid]["step"])
    assert res[0]["log"][0]["participants"] == [0, 1]
    assert any(e["participants"] == [0, 1, 2] for e in res[2]["log"])
    w = [torch.tensor(res[r]["weights"]) for r in (0, 1, 2)]
    assert torch.equal(w[0], w[1]) and torch.allclose(w[0], w[2], atol=0, rtol=0)


def _trainer_replica(rid, address, port, out):
    os.environ.update(RANK="0", LOCAL_RANK="0", WORLD_SIZE="1", MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.trainer import Trainer

    t = Trainer(ConfigManager().parse_args([
        "--module", "llama3", "--config", "llama3_debugmodel_cpu", "--training.steps", "4",
        "--training.seq-len", "64", "--metrics.log-freq", "1", "--dump-folder", os.path.join(out, f"r{rid}"),
        "--fault-tolerance.enable", "--fault-tolerance.lighthouse", address,
        "--fault-tolerance.replica-id", str(rid), "--fault-tolerance.group-size", "2",
        "--fault-tolerance.min-replica-size", "2", "--fault-tolerance.quorum-timeout-s", "20",
        "--fault-tolerance.process-group-timeout-ms", "60000"]))
    t.ft.store.set(f"ready/{rid}", "1")
    t.ft.store.wait(["ready/0", "ready/1"])
    t.train()
    flat = torch.cat([(p.full_tensor() if hasattr(p, "full_tensor") else p).detach().reshape(-1)
                      for p in t.model_parts[0].parameters()])
    torch.save({"w": flat.clone(), "step": t.step}, os.path.join(out, f"w{rid}.pt"))
    t.close()
    import torch.distributed as dist

    dist.destroy_process_group()


def test_trainer_replicas_train_in_lockstep():
    """Two single-process replica jobs of the Llama-3 debug model through the Trainer: each has
    its own default group and data shard, gradients are averaged across replicas every step, so
    both end with the same weights."""
    import socket

    from torchtitan_b200.parallel.ft import Lighthouse

    def port():
        s = socket.socket()
        s.bind(("127.0.0.1", 0))
        p = s.getsockname()[1]
        s.close()
        return p

    lh = Lighthouse(0)
    ctx = mp.get_context("spawn")
    with tempfile.TemporaryDirectory() as d:
        procs = [ctx.Process(target=_trainer_replica, args=(r, lh.address, port(), d)) for r in (0, 1)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=300)
            assert p.exitcode == 0
        w = [torch.load(os.path.join(d, f"w{r}.pt")) for r in (0, 1)]
    assert w[0]["step"] == w[1]["step"] == 4
    assert torch.equal(w[0]["w"], w[1]["w"])


def test_membership_run_start_is_the_same_for_every_participant():
    """The first round of a membership run comes from the store's closed lists, so a replica
    that missed rounds (and so never saw the membership change) agrees with one that took part
    in every round; both then build the cross-replica group under the same prefix."""
    from torchtitan_b200.parallel.ft import FTManager, Lighthouse

    lh = Lighthouse(0)
    for r, parts in enumerate(["0,1", "0,1", "1,2", "0,1", "0,1"]):
        lh.store.set(f"q/{r}/closed", parts)
    steady = FTManager(lh.address, 0, 3)
    late = FTManager(lh.address, 1, 3)
    # the steady replica walked through rounds 0..4; the late one only sees round 4
    assert [steady._membership_since(r, [int(x) for x in p.split(",")])
            for r, p in enumerate(["0,1", "0,1", "1,2", "0,1", "0,1"])] == [0, 0, 2, 3, 3]
    assert late._membership_since(4, [0, 1]) == 3
