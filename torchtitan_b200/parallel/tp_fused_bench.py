"""Fused TP GEMMs vs NCCL collective + GEMM, device-timed, max over ranks.

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        -m torchtitan_b200.parallel.tp_fused_bench

Shapes: Llama-3 70B TP linears at seq 8192 (hidden 8192, FFN 28672 sharded over N ranks):
column-parallel w1 (AG -> GEMM) and row-parallel w2 (GEMM -> RS). Roofline of a fused call is
the slower of its GEMM at the measured bf16 peak and its NVLink bytes at the measured peer
copy bandwidth (770 GB/s per direction per GPU).
"""
from __future__ import annotations

import json
import os

import torch
import torch.distributed as dist

PEAK_TFLOPS = 1674.7  # measured cuBLAS bf16 burst on this pool
LINK_GBS = 770.0


def _time(fn, iters=10, warmup=3):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    t = torch.tensor([s.elapsed_time(e) / iters], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t)


def main():
    rank = int(os.environ["RANK"])
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dist.init_process_group("nccl")
    tp = dist.get_world_size()
    from torchtitan_b200 import ops
    from torchtitan_b200.parallel import tp_fused

    g = dist.group.WORLD
    S, H, F = 8192, 8192, 28672
    Ms, Fl = S // tp, F // tp
    x = torch.randn(1, Ms, H, device="cuda").bfloat16()
    w1 = (torch.randn(Fl, H, device="cuda") * 0.02).bfloat16()
    xr = torch.randn(1, S, Fl, device="cuda").bfloat16()
    w2 = (torch.randn(H, Fl, device="cuda") * 0.02).bfloat16()
    c = tp_fused._comm(g)
    res = []
    # AG -> GEMM
    fused = _time(lambda: c.ag_gemm(x.view(Ms, H), w1, False))

    def nccl_ag():
        full = torch.empty(S, H, device="cuda", dtype=torch.bfloat16)
        dist.all_gather_into_tensor(full, x.view(Ms, H))
        return ops.linear(full, w1)

    base = _time(nccl_ag)
    flops = 2.0 * S * Fl * H
    link = (tp - 1) * Ms * H * 2
    roof = max(flops / (PEAK_TFLOPS * 1e12), link / (LINK_GBS * 1e9)) * 1e3
    res.append({"op": "ag_gemm", "tp": tp, "M": S, "N": Fl, "K": H, "fused_ms": fused, "nccl_then_gemm_ms": base,
                "roofline_ms": roof, "fraction_of_roofline": roof / fused, "speedup": base / fused})
    # GEMM -> RS
    fused = _time(lambda: c.gemm_rs(xr.view(S, Fl), w2, False))

    def nccl_rs():
        y = ops.linear(xr.view(S, Fl), w2)
        out = torch.empty(Ms, H, device="cuda", dtype=torch.bfloat16)
        dist.reduce_scatter_tensor(out, y)
        return out

    base = _time(nccl_rs)
    flops = 2.0 * S * H * Fl
    link = (tp - 1) * Ms * H * 2
    roof = max(flops / (PEAK_TFLOPS * 1e12), link / (LINK_GBS * 1e9)) * 1e3
    res.append({"op": "gemm_rs", "tp": tp, "M": S, "N": H, "K": Fl, "fused_ms": fused, "gemm_then_nccl_ms": base,
                "roofline_ms": roof, "fraction_of_roofline": roof / fused, "speedup": base / fused})
    from torchtitan_b200.ops._ext import ext

    res.append({"error_code": ext().tp_gemm_error_code(True)})
    if rank == 0:
        for r in res:
            print(json.dumps(r), flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
