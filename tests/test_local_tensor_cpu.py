"""``comm.mode=local_tensor``: one process simulates every rank of a TP = 2 mesh with
LocalTensorMode on a fake process group (reference: ``distributed/utils.py:296-336``), and its
training losses (same weights, same data) match the same TP = 2 run on two gloo processes."""
import os
import subprocess
import sys
import textwrap

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

_SCRIPT = textwrap.dedent("""
    import os, sys, zlib
    import torch
    from torch.distributed.tensor import DTensor, distribute_tensor
    if "LOCAL_WORLD_SIZE" not in os.environ:  # not launched by torchrun: one simulating process
        os.environ.update(WORLD_SIZE=sys.argv[1], RANK="0", LOCAL_RANK="0", MASTER_ADDR="127.0.0.1",
                          MASTER_PORT=sys.argv[2])
    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.trainer import Trainer
    t = Trainer(ConfigManager().parse_args(["--module", "llama3", "--config", "llama3_debugmodel",
        "--training.steps", "2", "--training.seq-len", "64", "--training.local-batch-size", "2",
        "--training.mixed-precision-param", "float32", "--metrics.log-freq", "1",
        "--dump-folder", sys.argv[3], *sys.argv[4:]]))
    # identical weights in both runs: the simulated ranks draw random init from their own
    # generator, so the test writes every parameter from a seed of its name
    try:
        from torch.distributed._local_tensor import maybe_disable_local_tensor_mode
    except ImportError:
        import contextlib
        maybe_disable_local_tensor_mode = contextlib.nullcontext
    with torch.no_grad():
        for n, p in t.model_parts[0].named_parameters():
            with maybe_disable_local_tensor_mode():
                g = torch.Generator().manual_seed(zlib.crc32(n.encode()))
                full = torch.randn(p.shape, generator=g) * 0.02 + (1.0 if "norm" in n else 0.0)
            p.copy_(distribute_tensor(full, p.device_mesh, p.placements) if isinstance(p, DTensor) else full)
    t.train()
    if int(os.environ["RANK"]) == 0:
        print("LOSS", t.metrics_processor.last_metrics["loss_metrics/global_avg_loss"])
""")


def _run(tmp_path, ws, port, *extra, procs=1):
    env = dict(os.environ, PYTHONPATH=ROOT, CUDA_VISIBLE_DEVICES="")
    script = tmp_path / "run.py"
    script.write_text(_SCRIPT)
    launch = [sys.executable]
    if procs > 1:
        launch += ["-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={procs}",
                   "--master-addr=127.0.0.1", f"--master-port={port}"]
    r = subprocess.run([*launch, str(script), str(ws), str(port), str(tmp_path / f"d{ws}{procs}"), *extra],
                       capture_output=True, text=True, env=env, timeout=600, cwd=ROOT)
    return r


def _loss(r):
    lines = [l for l in r.stdout.splitlines() if l.startswith("LOSS")]
    assert r.returncode == 0 and lines, r.stderr[-3000:]
    return float(lines[-1].split()[1])


def test_local_tensor_tp_matches_two_gloo_ranks(tmp_path):
    tp = ["--parallelism.data-parallel-shard-degree", "1", "--parallelism.tensor-parallel-degree", "2"]
    real = _loss(_run(tmp_path, 2, 29631, *tp, procs=2))
    simulated = _loss(_run(tmp_path, 2, 29632, "--comm.mode", "local_tensor", *tp))
    assert abs(real - simulated) < 1e-4 * abs(real), (real, simulated)


def test_local_tensor_rejects_fsdp_with_a_clear_error(tmp_path):
    r = _run(tmp_path, 2, 29633, "--comm.mode", "local_tensor", "--parallelism.data-parallel-shard-degree", "2")
    assert r.returncode != 0 and "local_tensor with FSDP" in r.stderr, r.stderr[-2000:]
