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
