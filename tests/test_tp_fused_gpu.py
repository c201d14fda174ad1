"""Fused tensor-parallel GEMMs (``csrc/tp_gemm.cu`` through ``parallel/tp_fused.py``) on 2 GPUs
against NCCL collectives around fp32 PyTorch matmuls: AG->GEMM and GEMM->RS, outputs and the
gradients of input and weight, for one and two batch rows, three calls in a row (so both
receive-buffer parities and advancing epochs are exercised)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")]


def _rel(a, b):
    return float((a.float() - b.float()).norm() / (b.float().norm() + 1e-12))


def _worker(rank, world, port, out):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", device_id=torch.device("cuda", rank))
    from torchtitan_b200.ops._ext import ext
    from torchtitan_b200.parallel import tp_fused

    group = dist.group.WORLD
    errs = []
    for B, s, K, N in [(1, 256, 512, 768), (2, 128, 256, 512), (1, 256, 512, 768)]:
        g = torch.Generator(device="cuda").manual_seed(100 + rank)
        gw = torch.Generator(device="cuda").manual_seed(7)  # weights identical on both ranks
        x = (torch.randn(B, s, K, device="cuda", generator=g) * 0.5).bfloat16().requires_grad_()
        w = (torch.randn(N, K, device="cuda", generator=gw) * 0.05).bfloat16().requires_grad_()
        dy = torch.randn(B, s * world, N, device="cuda", generator=g).bfloat16()
        # AG -> GEMM
        y = tp_fused.FusedAGMatmul.apply(x, w, group)
        y.backward(dy)
        xs = [torch.empty_like(x) for _ in range(world)]
        dist.all_gather(xs, x.detach())
        xf = torch.cat(xs, 1).float().requires_grad_()
        wf = w.detach().float().requires_grad_()
        yr = xf @ wf.t()
        yr.backward(dy.float())
        dsum = xf.grad.clone()
        dist.all_reduce(dsum)  # every rank's output depends on every shard: sum over ranks
        dx_ref = dsum[:, rank * s:(rank + 1) * s]
        dwsum = wf.grad.clone()  # (weight gradients stay per rank: each rank's w is its own shard)
        errs.append(("ag_y", _rel(y, yr)))
        errs.append(("ag_dx", _rel(x.grad, dx_ref)))
        errs.append(("ag_dw", _rel(w.grad, dwsum)))
        # GEMM -> RS  (input: full sequence, local K shard)
        x2 = (torch.randn(B, s * world, K, device="cuda", generator=g) * 0.5).bfloat16().requires_grad_()
        w2 = (torch.randn(N, K, device="cuda", generator=g) * 0.05).bfloat16().requires_grad_()
        dz = torch.randn(B, s, N, device="cuda", generator=g).bfloat16()
        z = tp_fused.FusedMatmulRS.apply(x2, w2, group)
        z.backward(dz)
        x2f, w2f = x2.detach().float().requires_grad_(), w2.detach().float().requires_grad_()
        full = x2f @ w2f.t()
        red = full.detach().clone()
        dist.all_reduce(red)
        zr = red[:, rank * s:(rank + 1) * s]
        dzs = [torch.empty_like(dz) for _ in range(world)]
        dist.all_gather(dzs, dz)
        full.backward(torch.cat(dzs, 1).float())
        errs.append(("rs_z", _rel(z, zr)))
        errs.append(("rs_dx", _rel(x2.grad, x2f.grad)))
        errs.append(("rs_dw", _rel(w2.grad, w2f.grad)))
    torch.cuda.synchronize()
    code = ext().tp_gemm_error_code(True)
    torch.save({"errs": errs, "code": code}, os.path.join(out, f"r{rank}.pt"))
    if rank == 0:
        print(errs, flush=True)
    dist.destroy_process_group()


def test_fused_tp_gemms_match_collectives(tmp_path):
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    mp.spawn(_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        res = torch.load(tmp_path / f"r{r}.pt")
        assert res["code"] == 0, res
        bad = [(n, e) for n, e in res["errs"] if e > 2e-2]
        assert not bad, (r, bad)


def _trainer(rank, world, port, out):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.ops._ext import ext
    from torchtitan_b200.parallel import async_tp, tp_fused
    from torchtitan_b200.trainer import Trainer

    res = []
    for extra in ([], ["--parallelism.enable-async-tensor-parallel"]):
        t = Trainer(ConfigManager().parse_args([
            "--module", "llama3", "--config", "llama3_debugmodel", "--training.steps", "3",
            "--training.seq-len", "512", "--training.local-batch-size", "1",
            "--parallelism.tensor-parallel-degree", "2", "--parallelism.data-parallel-shard-degree", "1",
            "--activation-checkpoint.mode", "none", "--metrics.log-freq", "1", "--debug.seed", "0",
            "--dump-folder", os.path.join(out, str(len(extra))), *extra]))
        calls = []
        if extra:  # count that the fused kernels, not the ring, carried the TP linears
            orig = tp_fused._GroupComm.ag_gemm
            tp_fused._GroupComm.ag_gemm = lambda self, *a, **k: (calls.append(1), orig(self, *a, **k))[1]
        t.train()
        res.append(t.metrics_processor.last_metrics["loss_metrics/global_avg_loss"])
        t.close()
        if extra:
            tp_fused._GroupComm.ag_gemm = orig
            res.append(len(calls))
    async_tp.ENABLED = False
    torch.cuda.synchronize()
    res.append(ext().tp_gemm_error_code(True))
    torch.save(res, os.path.join(out, f"t{rank}.pt"))
    dist.destroy_process_group()


def test_trainer_async_tp_on_fused_kernels_matches_sync_tp(tmp_path):
    """The Llama-3 debug model with TP = 2 and sequence parallelism: three training steps with the
    TP linears on the fused kernels match the same steps on NCCL collectives (bf16 tolerance)."""
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    mp.spawn(_trainer, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    sync_loss, fused_loss, calls, code = torch.load(tmp_path / "t0.pt")
    assert code == 0 and calls > 0, (calls, code)
    assert abs(sync_loss - fused_loss) < 2e-2 * abs(sync_loss), (sync_loss, fused_loss)


def _ulysses_trainer(rank, world, port, out):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.ops._ext import ext
    from torchtitan_b200.parallel import tp_fused
    from torchtitan_b200.trainer import Trainer

    res = []
    for flag in ("0", "1"):
        os.environ["TTB_ULYSSES_FUSED"] = flag
        t = Trainer(ConfigManager().parse_args([
            "--module", "llama3", "--config", "llama3_debugmodel", "--training.steps", "3",
            "--training.seq-len", "512", "--training.local-batch-size", "1",
            "--parallelism.context-parallel-degree", "2", "--parallelism.context-parallel-method", "ulysses",
            "--parallelism.data-parallel-shard-degree", "1",
            "--activation-checkpoint.mode", "none", "--metrics.log-freq", "1", "--debug.seed", "0",
            "--dump-folder", os.path.join(out, flag)]))
        calls = []
        orig = tp_fused._GroupComm.ag_gemm
        tp_fused._GroupComm.ag_gemm = lambda self, *a, **k: (calls.append(1), orig(self, *a, **k))[1]
        t.train()
        tp_fused._GroupComm.ag_gemm = orig
        res.append(t.metrics_processor.last_metrics["loss_metrics/global_avg_loss"])
        res.append(len(calls))
        t.close()
    torch.cuda.synchronize()
    res.append(ext().tp_gemm_error_code(True))
    torch.save(res, os.path.join(out, f"u{rank}.pt"))
    dist.destroy_process_group()


def test_ulysses_on_fused_kernels_matches_all_to_all(tmp_path):
    """Llama-3 debug model, Ulysses CP = 2: three training steps with the head sharding carried
    by the fused AG->GEMM / GEMM->RS kernels match the all-to-all formulation (bf16 tolerance)."""
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    mp.spawn(_ulysses_trainer, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    a2a_loss, a2a_calls, fused_loss, fused_calls, code = torch.load(tmp_path / "u0.pt")
    assert code == 0 and a2a_calls == 0 and fused_calls > 0, (a2a_calls, fused_calls, code)
    assert abs(a2a_loss - fused_loss) < 2e-2 * abs(a2a_loss), (a2a_loss, fused_loss)
