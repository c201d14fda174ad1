"""Compare the loss curves of two training runs (parity: reference
``scripts/loss_compare.py:63-1205``, which builds two commits and trains each
from the same seed checkpoint).

    python -m torchtitan_b200.loss_compare --baseline "<train args>" --test "<train args>" \\
        [--steps 10] [--assert-equal | --rtol 1e-4] [--ngpus 1]

Each side runs ``python -m torchtitan_b200.train <args>`` (through
``torch.distributed.run`` when ``--ngpus > 1``) with the same seed,
deterministic mode and JSONL metrics, then the per-step
``loss_metrics/global_avg_loss`` values are compared.  ``--assert-equal``
requires bit-identical losses; otherwise relative tolerance ``--rtol``.
"""
from __future__ import annotations

import argparse
import json
import os
import shlex
import subprocess
import sys
import tempfile

KEY = "loss_metrics/global_avg_loss"


def read_losses(dump_folder: str) -> dict[int, float]:
    path = os.path.join(dump_folder, "tb", "rank_0", "metrics.jsonl")
    out = {}
    with open(path) as f:
        for line in f:
            rec = json.loads(line)
            if KEY in rec:
                out[int(rec["step"])] = rec[KEY]
    return out


def run(args: str, steps: int, dump: str, ngpus: int, seed: int) -> dict[int, float]:
    base = [sys.executable, "-m"]
    if ngpus > 1:
        base += ["torch.distributed.run", "--standalone", "--nproc-per-node", str(ngpus), "-m"]
    cmd = base + ["torchtitan_b200.train", *shlex.split(args), "--training.steps", str(steps),
                  "--metrics.log-freq", "1", "--metrics.enable-jsonl", "--dump-folder", dump,
                  "--debug.seed", str(seed), "--debug.deterministic"]
    # a fresh job: no rendezvous settings inherited from the calling process
    env = {k: v for k, v in os.environ.items()
           if k not in ("RANK", "LOCAL_RANK", "WORLD_SIZE", "LOCAL_WORLD_SIZE", "MASTER_ADDR", "MASTER_PORT",
                        "GROUP_RANK", "ROLE_RANK", "TORCHELASTIC_RUN_ID")}
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))  # so the child imports this package
    env["PYTHONPATH"] = root + (os.pathsep + env["PYTHONPATH"] if env.get("PYTHONPATH") else "")
    subprocess.run(cmd, check=True, env=env)
    return read_losses(dump)


def compare(a: dict[int, float], b: dict[int, float], assert_equal: bool, rtol: float) -> list[str]:
    errs = []
    for step in sorted(set(a) | set(b)):
        if step not in a or step not in b:
            errs.append(f"step {step}: logged by one run only")
            continue
        x, y = a[step], b[step]
        bad = (x != y) if assert_equal else abs(x - y) > rtol * max(abs(x), abs(y), 1e-12)
        if bad:
            errs.append(f"step {step}: baseline {x!r} test {y!r}")
    return errs


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--baseline", required=True)
    ap.add_argument("--test", required=True)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--ngpus", type=int, default=1)
    ap.add_argument("--seed", type=int, default=42)
    ap.add_argument("--assert-equal", action="store_true")
    ap.add_argument("--rtol", type=float, default=1e-4)
    ap.add_argument("--output-folder", default=None)
    a = ap.parse_args(argv)
    root = a.output_folder or tempfile.mkdtemp(prefix="loss_compare_")
    la = run(a.baseline, a.steps, os.path.join(root, "baseline"), a.ngpus, a.seed)
    lb = run(a.test, a.steps, os.path.join(root, "test"), a.ngpus, a.seed)
    for s in sorted(la):
        print(f"step {s:4d}  baseline {la[s]:.6f}  test {lb.get(s, float('nan')):.6f}")
    errs = compare(la, lb, a.assert_equal, a.rtol)
    for e in errs:
        print("MISMATCH", e)
    return 1 if errs else 0


if __name__ == "__main__":
    sys.exit(main())
