"""Fault-tolerant replica groups with a per-step quorum (what the reference gets from TorchFT:
``experiments/ft/manager.py:36-227`` -- lighthouse, ``min_replica_size``, replicas that leave
and rejoin; torchft itself is not in this image).

Each *replica* is an independent job (its own ranks, its own default process group, its own
FSDP/TP layout). Replicas only meet through a *lighthouse*: a TCP key-value store that no
replica owns (``python -m torchtitan_b200.parallel.ft --port P`` or :class:`Lighthouse`).
Every step:

1. **Quorum.** The leader (local rank 0) of every live replica announces itself for the step.
   Once all replicas seen in the previous quorum have announced, or ``quorum_timeout_s`` has
   passed, the first leader to get there *closes* the quorum with an atomic compare-and-set;
   every leader reads the closed participant list, so all agree even if a replica arrives late
   (it waits for the next step). Fewer than ``min_replica_size`` participants is an error.
   Leaders pass the result to their replica's other ranks over the replica's own group.
2. **Heal.** A participant whose training step is behind the most advanced participant
   (a replica that restarted) receives the model and optimizer state from that participant
   before computing anything.
3. **Cross-replica reduction.** Rank ``r`` of every participating replica joins a gloo or NCCL
   group built for exactly this participant set (a fresh prefix of the lighthouse store per
   quorum, so a group never includes a replica that has gone); gradients are averaged there.
4. **Commit.** Every participant votes whether its step succeeded (a collective that timed out
   because a replica died mid-step votes no); the optimizer step is applied only if all vote
   yes, otherwise every participant drops the step and the next quorum excludes the dead one.

All waits are bounded; a replica that stops answering is left out of the next quorum instead
of hanging the others.
"""
from __future__ import annotations

import argparse
import datetime
import time
from dataclasses import dataclass

import torch
import torch.distributed as dist
import torch.nn as nn


@dataclass
class Quorum:
    step: int
    qid: int
    participants: list[int]   # replica ids, sorted
    source: int               # the most advanced participant (state donor for healing)
    behind: list[int]         # participants whose step is behind the source's
    source_step: int = 0      # the source's completed step count (what a healed replica adopts)
    since: int = 0            # first round of the unbroken run of rounds with these participants

    @property
    def size(self) -> int:
        return len(self.participants)


class Lighthouse:
    """The store every replica leader talks to (owned by no replica)."""

    def __init__(self, port: int = 0, host: str = "127.0.0.1"):
        self.store = dist.TCPStore(host, port, is_master=True, wait_for_workers=False,
                                   timeout=datetime.timedelta(seconds=60))
        self.host, self.port = host, self.store.port

    @property
    def address(self) -> str:
        return f"{self.host}:{self.port}"


def _client(address: str, timeout_s: float) -> dist.TCPStore:
    host, port = address.rsplit(":", 1)
    return dist.TCPStore(host, int(port), is_master=False, timeout=datetime.timedelta(seconds=timeout_s))


class FTManager:
    """Quorum, healing, cross-replica reduction and commit votes for one rank of one replica."""

    def __init__(self, lighthouse: str, replica_id: int, group_size: int, *, min_replica_size: int = 1,
                 quorum_timeout_s: float = 5.0, collective_timeout_s: float = 10.0, backend: str = "gloo",
                 local_group=None):
        if not 0 <= replica_id < group_size:
            raise ValueError(f"replica_id {replica_id} outside [0, {group_size})")
        self.store = _client(lighthouse, max(quorum_timeout_s, collective_timeout_s) * 4)
        self.replica_id, self.group_size = replica_id, group_size
        self.min_replica_size = min_replica_size
        self.quorum_timeout_s, self.collective_timeout_s = quorum_timeout_s, collective_timeout_s
        self.backend = backend
        self.local_group = local_group  # this replica's own group (None: the default group, if any)
        live = dist.is_initialized()
        self.local_rank = dist.get_rank(local_group) if live else 0
        self.local_world = dist.get_world_size(local_group) if live else 1
        self._pgs: dict[tuple, dist.ProcessGroup] = {}
        self._retired: list[dist.ProcessGroup] = []
        self._last: list[int] = []
        self._closed_seen: dict[int, str] = {}  # round -> closed participant list (store values)
        self._since_seen: dict[int, int] = {}   # round -> first round of its membership run
        self._round: int | None = None  # quorum rounds are numbered by the lighthouse, not by steps
        self._fresh = True  # never synchronised with another replica: copy state at the first quorum
        self.quorum: Quorum | None = None

    # ------------------------------------------------------------------ quorum
    def _next_round(self) -> int:
        """After the last closed round: where a new or restarted replica joins."""
        s = self.store
        return int(s.get("latest").decode()) + 1 if s.check(["latest"]) else 0

    def _leader_quorum(self, my_step: int) -> tuple[int, list[int], dict[int, int]]:
        s = self.store
        deadline_all = time.monotonic() + 4 * self.quorum_timeout_s
        while True:
            if self._round is None:
                self._round = self._next_round()
            rnd = self._round
            qid, parts, steps = self._leader_round(rnd, my_step)
            if self.replica_id in parts or time.monotonic() > deadline_all:
                return qid, parts, steps
            self._round = None  # arrived after that round closed: join the next one
            self._last = []

    def _leader_round(self, step: int, my_step: int) -> tuple[int, list[int], dict[int, int]]:
        s = self.store
        s.set(f"q/{step}/join/{self.replica_id}", f"{my_step},{int(self._fresh)}")
        expected = set(self._last) | {self.replica_id}
        deadline = time.monotonic() + self.quorum_timeout_s
        closed = None
        while closed is None:
            joined = [r for r in range(self.group_size) if s.check([f"q/{step}/join/{r}"])]
            if s.check([f"q/{step}/closed"]):
                closed = s.get(f"q/{step}/closed").decode()
                break
            now = time.monotonic()
            enough = len(joined) >= self.min_replica_size
            # close when everyone of the last quorum is back, or after the timeout; never below
            # the minimum size unless even a long wait (four timeouts) brought no one else
            if (enough and (expected.issubset(joined) or now > deadline)) or now > deadline + 3 * self.quorum_timeout_s:
                proposal = ",".join(str(r) for r in sorted(joined))
                got = s.compare_set(f"q/{step}/closed", "", proposal).decode()
                closed = got if got else proposal
                if closed == proposal:
                    s.set("latest", str(step))
                break
            time.sleep(0.005)
        participants = [int(x) for x in closed.split(",") if x]
        steps = {r: tuple(int(x) for x in s.get(f"q/{step}/join/{r}").decode().split(",")) for r in participants}
        return step, participants, steps  # one quorum per round: the round is its id

    def _membership_since(self, qid: int, parts: list[int]) -> int:
        """First round of the unbroken run of closed rounds ending at ``qid`` whose participants
        equal ``parts``.  Computed from the store's closed lists, which never change, so every
        participant gets the same answer whichever earlier rounds it took part in."""
        s = self.store
        closed = ",".join(str(r) for r in parts)
        r = qid
        while r > 0:
            prev = self._closed_seen.get(r - 1)
            if prev is None:
                if not s.check([f"q/{r - 1}/closed"]):
                    break
                prev = s.get(f"q/{r - 1}/closed").decode()
                self._closed_seen[r - 1] = prev
            if prev != closed:
                break
            if (r - 1) in self._since_seen:
                r = self._since_seen[r - 1]
                break
            r -= 1
        self._closed_seen[qid] = closed
        self._since_seen[qid] = r
        return r

    def start_quorum(self, my_step: int) -> Quorum:
        """Form (or learn) the next quorum; ``my_step`` is this replica's completed step count
        (what healing compares). A replica that arrives after a round closed joins the next
        one. Raises if fewer than ``min_replica_size`` replicas joined."""
        if self.local_rank == 0:
            qid, parts, steps = self._leader_quorum(my_step)
            self._round = qid + 1
            payload = [qid, parts, steps, self._membership_since(qid, parts)]
        else:
            payload = [None, None, None, None]
        if self.local_world > 1:
            dist.broadcast_object_list(payload, src=dist.get_global_rank(self.local_group, 0)
                                       if self.local_group is not None else 0, group=self.local_group)
        qid, parts, steps, since = payload
        if self.replica_id not in parts:
            raise RuntimeError(f"replica {self.replica_id} found no quorum to join (last: {parts})")
        if len(parts) < self.min_replica_size:
            raise RuntimeError(f"quorum {qid} has {len(parts)} replicas, fewer than the minimum "
                               f"{self.min_replica_size}")
        # source: the most advanced replica, preferring ones that already trained with others;
        # behind: replicas with fewer steps, and replicas in their first quorum (fresh weights)
        best = max(parts, key=lambda r: (steps[r][0], 1 - steps[r][1], -r))
        behind = [r for r in parts if r != best and (steps[r][0] < steps[best][0] or steps[r][1])]
        self._last = parts
        self._fresh = False
        self.quorum = Quorum(qid, qid, parts, best, behind, steps[best][0], since)
        return self.quorum

    @property
    def healing(self) -> bool:
        return self.quorum is not None and self.replica_id in self.quorum.behind

    # ------------------------------------------------------------------ cross-replica group
    def replica_group(self) -> dist.ProcessGroup | None:
        """The group of this rank's peers (same local rank) in the current quorum's replicas."""
        q = self.quorum
        assert q is not None, "start_quorum first"
        if q.size == 1:
            return None
        # one group per run of rounds with the same participants: reused within the run, rebuilt
        # (under the prefix of the run's first round) when it changes.  The run's first round
        # comes from the store, not from this replica's history: a replica that missed a round
        # (arrived after it closed) must not reuse a group its peers have replaced.
        key = (q.since, tuple(q.participants))
        pg = self._pgs.get(key)
        if pg is None:
            prefix = dist.PrefixStore(f"pg/{q.since}/{','.join(map(str, q.participants))}/{self.local_rank}",
                                      self.store)
            rank = q.participants.index(self.replica_id)
            timeout = datetime.timedelta(seconds=self.collective_timeout_s)
            if self.backend == "gloo":
                pg = dist.ProcessGroupGloo(prefix, rank, q.size, timeout)
            else:
                opts = dist.ProcessGroupNCCL.Options()
                opts._timeout = timeout
                pg = dist.ProcessGroupNCCL(prefix, rank, q.size, opts)
            # older groups are kept, not destroyed: tearing down a group whose peer has died can
            # block on that peer; membership changes are rare, so the few retired groups are cheap
            self._retired.extend(self._pgs.values())
            self._pgs = {key: pg}
        return pg

    # ------------------------------------------------------------------ steps
    @torch.no_grad()
    def heal(self, modules: list[nn.Module], *statefuls) -> bool:
        """If a participant is behind, the most advanced one sends every parameter and buffer
        (tensor by tensor, same order everywhere) and the state dicts of ``statefuls``
        (optimizer, LR schedulers, ...) to all participants; the ones behind load them.
        Returns whether this replica healed."""
        q = self.quorum
        if q is None or q.size == 1 or not q.behind:
            return False
        # every participant knows the same source and the same set of replicas behind it
        pg = self.replica_group()
        src = q.participants.index(q.source)
        for t in _state_tensors(modules):
            pg.broadcast([t], _bopts(src)).wait()
        for obj in statefuls:
            # a restarted replica may hold no optimizer state yet (it is created on the first
            # step), so each state dict travels as one serialized blob rather than tensor by tensor
            import io

            dev = _device_of(modules)
            if self.replica_id == q.source:
                buf = io.BytesIO()
                torch.save(obj.state_dict(), buf)
                blob = torch.frombuffer(bytearray(buf.getvalue()), dtype=torch.uint8).to(dev)
                n = torch.tensor([blob.numel()], dtype=torch.int64, device=dev)
            else:
                n = torch.zeros(1, dtype=torch.int64, device=dev)
            pg.broadcast([n], _bopts(src)).wait()
            if self.replica_id != q.source:
                blob = torch.empty(int(n.item()), dtype=torch.uint8, device=dev)
            pg.broadcast([blob], _bopts(src)).wait()
            if self.healing:
                obj.load_state_dict(torch.load(io.BytesIO(blob.cpu().numpy().tobytes()), weights_only=False))
        return self.healing

    @torch.no_grad()
    def allreduce_gradients(self, modules: list[nn.Module]) -> bool:
        """Average gradients over the quorum's replicas (local shards: every replica shards its
        parameters the same way). Returns False if the collective failed (a replica died)."""
        pg = self.replica_group()
        if pg is None:
            return True
        grads = [p.grad for m in modules for p in m.parameters() if p.grad is not None]
        if not grads:
            return True
        locs = [g.to_local() if hasattr(g, "to_local") else g for g in grads]
        flat = torch.cat([x.reshape(-1).float() for x in locs])
        try:
            work = pg.allreduce([flat])
            work.wait()
        except Exception:  # noqa: BLE001 - a peer left mid-step; the commit vote drops the step
            return False
        flat /= self.quorum.size
        o = 0
        for x in locs:
            x.copy_(flat[o:o + x.numel()].view_as(x))
            o += x.numel()
        return True

    def should_commit(self, ok: bool) -> bool:
        """Every participant votes; the step is applied only if all voted yes within the limit."""
        q = self.quorum
        assert q is not None
        vote = torch.tensor([1 if ok else 0], dtype=torch.int32)
        if self.local_world > 1:  # a replica votes yes only if all its ranks do
            dist.all_reduce(vote, op=dist.ReduceOp.MIN, group=self.local_group)
        if self.local_rank == 0:
            s = self.store
            s.set(f"q/{q.step}/vote/{self.replica_id}", str(int(vote.item())))
            deadline = time.monotonic() + self.collective_timeout_s
            verdict = 1
            for r in q.participants:
                key = f"q/{q.step}/vote/{r}"
                while not s.check([key]):
                    if time.monotonic() > deadline:
                        verdict = 0
                        break
                    time.sleep(0.002)
                if verdict and s.check([key]) and s.get(key).decode() != "1":
                    verdict = 0
            decision = torch.tensor([verdict], dtype=torch.int32)
        else:
            decision = torch.tensor([0], dtype=torch.int32)
        if self.local_world > 1:
            dist.broadcast(decision, src=dist.get_global_rank(self.local_group, 0)
                           if self.local_group is not None else 0, group=self.local_group)
        return bool(decision.item())

    def data_parallel_info(self, dp_degree: int, dp_rank: int) -> tuple[int, int]:
        """Data sharding across replicas: (total data-parallel degree, this rank's index)."""
        return dp_degree * self.group_size, dp_degree * self.replica_id + dp_rank


def _bopts(root: int) -> "dist.BroadcastOptions":
    o = dist.BroadcastOptions()
    o.rootRank = root
    o.rootTensor = 0
    return o


def _device_of(modules: list[nn.Module]) -> torch.device:
    for m in modules:
        for p in m.parameters():
            return (p.to_local() if hasattr(p, "to_local") else p).device
    return torch.device("cpu")


def _state_tensors(modules: list[nn.Module]) -> list[torch.Tensor]:
    """Parameters (and their fp32 masters) and buffers, in a fixed order on every replica."""
    out = []
    for m in modules:
        for t in list(m.parameters()) + list(m.buffers()):
            x = t.to_local() if hasattr(t, "to_local") else t
            out.append(x.data)
            master = getattr(t, "_master", None)
            if master is not None:
                out.append(master)
    return out


def main() -> None:
    ap = argparse.ArgumentParser(description="fault-tolerance lighthouse: the store replica leaders meet at")
    ap.add_argument("--host", default="0.0.0.0")
    ap.add_argument("--port", type=int, default=29510)
    a = ap.parse_args()
    lh = Lighthouse(a.port, a.host)
    print(f"lighthouse listening on {lh.address}", flush=True)
    while True:
        time.sleep(3600)


if __name__ == "__main__":
    main()
