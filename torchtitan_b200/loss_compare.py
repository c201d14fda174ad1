"""Compare the loss curves of two training runs, across git revisions and/or training
configurations (parity: reference ``scripts/loss_compare.py:63-1205``).

    python -m torchtitan_b200.loss_compare BASELINE_REV TEST_REV \\
        [--baseline-module llama3] [--baseline-config llama3_debugmodel] [--baseline-options "..."] \\
        [--test-module ...] [--test-config ...] [--test-options "..."] \\
        [--steps 100] [--baseline-ngpus 1] [--test-ngpus 1] [--no-seed-checkpoint] \\
        [--assert-equal | --rtol 1e-4] [--export-result FILE] [--import-result FILE] \\
        [--output-folder DIR] [--build]

A revision is ``.`` (this working tree, as it is) or anything ``git rev-parse``
accepts.  A revision other than ``.`` is checked out into a temporary
``git worktree`` (the caller's tree is never touched) and, with ``--build``, its
CUDA extension is compiled there.  Unless ``--no-seed-checkpoint`` is given, the
baseline side first writes a seed checkpoint (one process, model only, full
precision) that both sides load, so their initial weights are identical even when
their parallel layouts differ.  Every run adds ``--debug.deterministic``, a fixed
seed and per-step JSONL metrics; the per-step ``loss_metrics/global_avg_loss``
values are then compared step by step, with average losses and the largest
difference.  ``--assert-equal`` demands bit-identical losses (the reference's CI
mode), otherwise ``--rtol`` bounds the relative difference.  ``--export-result``
writes ``step loss`` lines (``repr`` precision); ``--import-result`` adds a third,
recorded curve that both runs must match.  With ``--output-folder`` every run's log,
the seed checkpoint and a ``summary.txt`` are kept there.

Exit status: 0 when the curves agree, 1 otherwise.
"""
from __future__ import annotations

import argparse
import json
import os
import shlex
import shutil
import subprocess
import sys
import tempfile
from dataclasses import dataclass

KEY = "loss_metrics/global_avg_loss"
FIXED = ["--debug.deterministic", "--metrics.log-freq", "1", "--metrics.enable-jsonl"]
_RDZV_ENV = ("RANK", "LOCAL_RANK", "WORLD_SIZE", "LOCAL_WORLD_SIZE", "MASTER_ADDR", "MASTER_PORT",
             "GROUP_RANK", "ROLE_RANK", "TORCHELASTIC_RUN_ID")
HERE = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@dataclass
class Side:
    name: str
    rev: str
    module: str
    config: str
    options: str
    ngpus: int


# --------------------------------------------------------------------------- source trees
def _git(args: list[str], cwd: str) -> str:
    return subprocess.run(["git", *args], cwd=cwd, check=True, capture_output=True, text=True).stdout.strip()


class Trees:
    """Source trees per revision: ``.`` is this checkout; other revisions get a detached
    worktree under a temporary folder, removed on ``close``."""

    def __init__(self, build: bool):
        self.build = build
        self._tmp: str | None = None
        self._trees: dict[str, str] = {}

    def get(self, rev: str) -> str:
        if rev == ".":
            return HERE
        sha = _git(["rev-parse", "--verify", f"{rev}^{{commit}}"], HERE)
        if sha not in self._trees:
            self._tmp = self._tmp or tempfile.mkdtemp(prefix="loss_compare_trees_")
            path = os.path.join(self._tmp, sha[:12])
            _git(["worktree", "add", "--detach", path, sha], HERE)
            if self.build:
                subprocess.run([sys.executable, "setup.py", "build_ext", "--inplace"], cwd=path, check=True)
            self._trees[sha] = path
        return self._trees[sha]

    def close(self) -> None:
        for path in self._trees.values():
            subprocess.run(["git", "worktree", "remove", "--force", path], cwd=HERE, check=False,
                           capture_output=True)
        if self._tmp:
            shutil.rmtree(self._tmp, ignore_errors=True)


# --------------------------------------------------------------------------- runs
def _launch(tree: str, args: list[str], ngpus: int, log_path: str) -> None:
    cmd = [sys.executable, "-m"]
    if ngpus > 1:
        cmd += ["torch.distributed.run", "--nnodes=1", "--nproc-per-node", str(ngpus), "--master-addr",
                "127.0.0.1", "--master-port", str(_free_port()), "-m"]
    cmd += ["torchtitan_b200.train", *args]
    env = {k: v for k, v in os.environ.items() if k not in _RDZV_ENV}  # a fresh job
    env["PYTHONPATH"] = tree + (os.pathsep + env["PYTHONPATH"] if env.get("PYTHONPATH") else "")
    env["PYTHONUNBUFFERED"] = "1"
    print(f"[loss_compare] {' '.join(shlex.quote(c) for c in cmd)}  (log: {log_path})", flush=True)
    with open(log_path, "w") as log:
        r = subprocess.run(cmd, cwd=tree, env=env, stdout=log, stderr=subprocess.STDOUT)
    if r.returncode:
        with open(log_path) as f:
            tail = f.read()[-4000:]
        raise RuntimeError(f"training run failed (exit {r.returncode}); end of {log_path}:\n{tail}")


def _free_port() -> int:
    import socket

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _base_args(side: Side, dump: str, seed: int) -> list[str]:
    return ["--module", side.module, "--config", side.config, *shlex.split(side.options), *FIXED,
            "--debug.seed", str(seed), "--dump-folder", dump]


def create_seed_checkpoint(tree: str, side: Side, out: str, seed: int) -> str:
    dump = os.path.join(out, "seed")
    _launch(tree, _base_args(side, dump, seed) + ["--checkpoint.enable", "--checkpoint.create-seed-checkpoint"], 1,
            os.path.join(out, "seed_training.log"))
    return os.path.join(dump, "checkpoint", "step-0")


def run_side(tree: str, side: Side, out: str, steps: int, seed: int, seed_ckpt: str | None) -> dict[int, float]:
    dump = os.path.join(out, side.name)
    shutil.rmtree(os.path.join(dump, "tb"), ignore_errors=True)  # no stale metrics from an earlier run
    args = _base_args(side, dump, seed) + ["--training.steps", str(steps)]
    if seed_ckpt:
        args += ["--checkpoint.enable", "--checkpoint.load-only", "--checkpoint.initial-load-path", seed_ckpt]
    _launch(tree, args, side.ngpus, os.path.join(out, f"{side.name}_training.log"))
    return read_losses(dump)


def read_losses(dump_folder: str) -> dict[int, float]:
    path = os.path.join(dump_folder, "tb", "rank_0", "metrics.jsonl")
    out = {}
    with open(path) as f:
        for line in f:
            rec = json.loads(line)
            if KEY in rec:
                out[int(rec["step"])] = rec[KEY]
    return out


# --------------------------------------------------------------------------- results
def export_losses(losses: dict[int, float], path: str) -> None:
    with open(path, "w") as f:
        for s in sorted(losses):
            f.write(f"{s} {losses[s]!r}\n")


def import_losses(path: str) -> dict[int, float]:
    out = {}
    with open(path) as f:
        for line in f:
            if line.strip():
                s, v = line.split()
                out[int(s)] = float(v)
    return out


def compare(a: dict[int, float], b: dict[int, float], assert_equal: bool, rtol: float) -> list[str]:
    errs = []
    for step in sorted(set(a) | set(b)):
        if step not in a or step not in b:
            errs.append(f"step {step}: logged by one run only")
            continue
        x, y = a[step], b[step]
        bad = (x != y) if assert_equal else abs(x - y) > rtol * max(abs(x), abs(y), 1e-12)
        if bad:
            errs.append(f"step {step}: {x!r} vs {y!r}")
    return errs


def summary(curves: dict[str, dict[int, float]]) -> str:
    names = list(curves)
    steps = sorted(set().union(*(set(c) for c in curves.values())))
    lines = ["step  " + "  ".join(f"{n:>22}" for n in names) + ("  difference" if len(names) >= 2 else "")]
    for s in steps:
        vals = [curves[n].get(s) for n in names]
        row = f"{s:4d}  " + "  ".join(f"{v!r:>22}" if v is not None else f"{'-':>22}" for v in vals)
        if len(names) >= 2 and vals[0] is not None and vals[1] is not None:
            row += f"  {vals[1] - vals[0]:+.3e}"
        lines.append(row)
    for n in names:
        c = curves[n]
        if c:
            lines.append(f"average {n}: {sum(c.values()) / len(c)!r}")
    if len(names) >= 2:
        common = set(curves[names[0]]) & set(curves[names[1]])
        if common:
            worst = max(common, key=lambda s: abs(curves[names[1]][s] - curves[names[0]][s]))
            lines.append(f"largest difference: step {worst}, "
                         f"{curves[names[1]][worst] - curves[names[0]][worst]:+.3e}")
    return "\n".join(lines)


# --------------------------------------------------------------------------- CLI
def parse_args(argv: list[str] | None = None) -> argparse.Namespace:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0],
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("baseline_rev", nargs="?", default=".")
    ap.add_argument("test_rev", nargs="?", default=".")
    ap.add_argument("--baseline-module", default="llama3")
    ap.add_argument("--test-module", default="")
    ap.add_argument("--baseline-config", default="llama3_debugmodel")
    ap.add_argument("--test-config", default="")
    ap.add_argument("--baseline-options", default="")
    ap.add_argument("--test-options", default="")
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--seed", type=int, default=42)
    ap.add_argument("--baseline-ngpus", type=int, default=1)
    ap.add_argument("--test-ngpus", type=int, default=1)
    ap.add_argument("--no-seed-checkpoint", action="store_true")
    ap.add_argument("--assert-equal", action="store_true")
    ap.add_argument("--rtol", type=float, default=1e-4)
    ap.add_argument("--export-result", default="")
    ap.add_argument("--import-result", default="")
    ap.add_argument("--output-folder", default="")
    ap.add_argument("--build", action="store_true", help="compile the CUDA extension in each checked-out revision")
    ap.add_argument("--baseline-only", action="store_true",
                    help="run the baseline side alone (with --export-result or --import-result)")
    a = ap.parse_args(argv)
    a.test_module = a.test_module or a.baseline_module
    a.test_config = a.test_config or a.baseline_config
    if a.baseline_only and not (a.export_result or a.import_result):
        ap.error("--baseline-only needs --export-result or --import-result")
    return a


def main(argv: list[str] | None = None) -> int:
    a = parse_args(argv)
    keep = bool(a.output_folder)
    out = os.path.abspath(a.output_folder) if keep else tempfile.mkdtemp(prefix="loss_compare_")
    os.makedirs(out, exist_ok=True)
    base = Side("baseline", a.baseline_rev, a.baseline_module, a.baseline_config, a.baseline_options,
                a.baseline_ngpus)
    test = Side("test", a.test_rev, a.test_module, a.test_config, a.test_options, a.test_ngpus)
    trees = Trees(a.build)
    try:
        seed_ckpt = None
        if not a.no_seed_checkpoint:
            seed_ckpt = create_seed_checkpoint(trees.get(base.rev), base, out, a.seed)
        curves = {"baseline": run_side(trees.get(base.rev), base, out, a.steps, a.seed, seed_ckpt)}
        if not a.baseline_only:
            curves["test"] = run_side(trees.get(test.rev), test, out, a.steps, a.seed, seed_ckpt)
    finally:
        trees.close()
    if a.import_result:
        curves["imported"] = import_losses(a.import_result)
    text = summary(curves)
    print(text)
    errs = []
    names = list(curves)
    for other in names[1:]:
        errs += [f"baseline vs {other}: {e}" for e in compare(curves["baseline"], curves[other], a.assert_equal,
                                                              a.rtol)]
    for e in errs:
        print("MISMATCH", e)
    if keep:
        with open(os.path.join(out, "summary.txt"), "w") as f:
            f.write(text + "\n" + "\n".join(f"MISMATCH {e}" for e in errs) + "\n")
    if a.export_result and not errs:
        export_losses(curves["baseline"], a.export_result)
    if not keep:
        shutil.rmtree(out, ignore_errors=True)
    return 1 if errs else 0


if __name__ == "__main__":
    sys.exit(main())
