"""Kernel micro-benchmarks: ``python -m torchtitan_b200.ops.benchmark [--only gemm,attn,...]``.

Times each sm_100a kernel with CUDA events on the launching stream after
warm-up, flushing L2 (a 256 MB write) before every timed launch, and prints
one JSON line per case with the achieved TFLOP/s or GB/s next to the same
operation done by the library path (cuBLAS ``torch.matmul`` / torch SDPA)
on the same shapes.  Shapes are those of the Llama-3 8B benchmark config
(seq 8192, dim 4096, FFN 14336, vocab 128256, 32 heads / 8 KV heads).
"""
from __future__ import annotations

import argparse
import json
import math

import torch


def _flush(buf):
    buf.zero_()


def time_fn(fn, iters=10, warmup=3, flush=True):
    buf = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda") if flush else None
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        if buf is not None:
            _flush(buf)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        e.synchronize()
        times.append(s.elapsed_time(e))
    times.sort()
    return times[len(times) // 2]  # median ms


def bench_gemm(ext, out):
    shapes = [  # (name, M, N, K, a_mn, b_mn)
        ("qkv_fwd", 8192, 6144, 4096, False, False),
        ("w13_fwd", 8192, 28672, 4096, False, False),
        ("w2_fwd", 8192, 4096, 14336, False, False),
        ("w2_dgrad", 8192, 14336, 4096, False, True),
        ("w2_wgrad", 4096, 14336, 8192, True, True),
        ("out_fwd", 8192, 128256, 4096, False, False),
        ("sq8192", 8192, 8192, 8192, False, False),
    ]
    for name, M, N, K, amn, bmn in shapes:
        A = torch.randn((K, M) if amn else (M, K), device="cuda", dtype=torch.bfloat16)
        B = torch.randn((K, N) if bmn else (N, K), device="cuda", dtype=torch.bfloat16)
        ours = time_fn(lambda: ext.gemm(A, B, amn, bmn))
        ours2 = time_fn(lambda: ext.gemm_2sm(A, B, amn, bmn)) if hasattr(ext, "gemm_2sm") else float("nan")
        At = A.t() if amn else A
        Bt = B if bmn else B.t()
        lib = time_fn(lambda: torch.matmul(At, Bt))
        fl = 2.0 * M * N * K
        out.append({"kernel": "gemm_tcgen05", "case": name, "M": M, "N": N, "K": K, "ms": ours,
                    "tflops": fl / ours / 1e9, "tflops_2sm": fl / ours2 / 1e9, "cublas_ms": lib, "cublas_tflops": fl / lib / 1e9,
                    "ratio_vs_cublas": lib / ours, "err": ext.gemm_error_code(True) + ext.gemm2_error_code(True)})
        print(json.dumps(out[-1]), flush=True)


def bench_attn(ext, out):
    from torchtitan_b200 import ops

    for (B, S, H, Hk, D, Dv) in [(1, 8192, 32, 8, 128, 128), (2, 4096, 32, 32, 192, 128)]:
        q = torch.randn(B, S, H, D, device="cuda", dtype=torch.bfloat16)
        k = torch.randn(B, S, Hk, D, device="cuda", dtype=torch.bfloat16)
        v = torch.randn(B, S, Hk, Dv, device="cuda", dtype=torch.bfloat16)
        sc = 1 / math.sqrt(D)
        o, lse = ext.attn_fwd(q, k, v, True, sc)
        do = torch.randn_like(o)
        f_ms = time_fn(lambda: ext.attn_fwd(q, k, v, True, sc))
        b_ms = time_fn(lambda: ext.attn_bwd(do, q, k, v, o, lse, True, sc))
        # causal FLOPs (half of the full S x S)
        fwd_fl = 2.0 * B * H * S * S * (D + Dv) / 2
        bwd_fl = 2.0 * B * H * S * S * (2 * D + 3 * Dv) / 2  # dS K, dS^T Q, P^T dO, dO V^T, (S recompute counted)
        qt, kt, vt = (t.transpose(1, 2) for t in (q, k, v))
        try:
            lib_f = time_fn(lambda: torch.nn.functional.scaled_dot_product_attention(qt, kt, vt, is_causal=True,
                                                                                     enable_gqa=True, scale=sc))
        except Exception as e:  # noqa: BLE001
            lib_f = float("nan")
        rec = {"kernel": "flash_attn_tcgen05", "B": B, "S": S, "H": H, "Hk": Hk, "D": D, "Dv": Dv,
               "fwd_ms": f_ms, "fwd_tflops": fwd_fl / f_ms / 1e9, "bwd_ms": b_ms, "bwd_tflops": bwd_fl / b_ms / 1e9,
               "sdpa_fwd_ms": lib_f, "sdpa_fwd_tflops": fwd_fl / lib_f / 1e9, "err": ext.attn_error_code(True)}
        out.append(rec)
        print(json.dumps(rec), flush=True)


def bench_memory_bound(ext, out):
    from torchtitan_b200 import ops

    T, Dm, V = 8192, 4096, 128256
    x = torch.randn(T, Dm, device="cuda", dtype=torch.bfloat16)
    w = torch.ones(Dm, device="cuda", dtype=torch.bfloat16)
    # rows x 4096: 8192 rows (64 MB, the 8B step's shape) and 65536 rows (512 MB, well above
    # L2, so the dirty lines of the L2 flush no longer dominate)
    for rows in (T, 8 * T):
        xr = torch.randn(rows, Dm, device="cuda", dtype=torch.bfloat16)
        ms = time_fn(lambda: ext.rmsnorm_fwd(xr, w, 1e-5))
        out.append({"kernel": "rmsnorm_fwd", "rows": rows, "ms": ms, "gbs": 2 * xr.numel() * 2 / ms / 1e6})
        print(json.dumps(out[-1]), flush=True)
        _, rstd = ext.rmsnorm_fwd(xr, w, 1e-5)
        dy = torch.randn_like(xr)
        ms = time_fn(lambda: ext.rmsnorm_bwd(dy, xr, w, rstd))
        out.append({"kernel": "rmsnorm_bwd", "rows": rows, "ms": ms, "gbs": 3 * xr.numel() * 2 / ms / 1e6})
        print(json.dumps(out[-1]), flush=True)
        del xr, dy
    a = torch.randn(T, 14336, device="cuda", dtype=torch.bfloat16)
    b = torch.randn_like(a)
    ms = time_fn(lambda: ext.swiglu_fwd(a, b))
    out.append({"kernel": "swiglu_fwd", "ms": ms, "gbs": 3 * a.numel() * 2 / ms / 1e6})
    print(json.dumps(out[-1]), flush=True)
    logits = torch.randn(T, V, device="cuda", dtype=torch.bfloat16)
    labels = torch.randint(0, V, (T,), device="cuda")
    ms = time_fn(lambda: ext.ce_fwd(logits, labels, -100))
    out.append({"kernel": "ce_fwd", "ms": ms, "gbs": logits.numel() * 2 / ms / 1e6})
    print(json.dumps(out[-1]), flush=True)
    loss, lse = ext.ce_fwd(logits, labels, -100)
    g = torch.ones(1, device="cuda")
    ms = time_fn(lambda: ext.ce_bwd(logits, labels, lse, g, -100))
    out.append({"kernel": "ce_bwd", "ms": ms, "gbs": 2 * logits.numel() * 2 / ms / 1e6})
    print(json.dumps(out[-1]), flush=True)
    n = 256 * 1024 * 1024
    p = torch.randn(n, device="cuda")
    gr = torch.randn(n, device="cuda")
    m = torch.zeros(n, device="cuda")
    vv = torch.zeros(n, device="cuda")
    ms = time_fn(lambda: ext.adamw([p], [gr], [m], [vv], 1e-3, 0.9, 0.95, 1e-8, 0.1, 1))
    out.append({"kernel": "adamw", "ms": ms, "gbs": n * 4 * 7 / ms / 1e6})
    print(json.dumps(out[-1]), flush=True)


def small_cases(ext, out):
    """A few launches of each kernel on small shapes (for ncu captures)."""
    B, S, H, Hk, D = 1, 2048, 8, 8, 128
    q = torch.randn(B, S, H, D, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(B, S, Hk, D, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(B, S, Hk, D, device="cuda", dtype=torch.bfloat16)
    for _ in range(2):
        o, lse = ext.attn_fwd(q, k, v, True, 1 / math.sqrt(D))
        ext.attn_bwd(torch.randn_like(o), q, k, v, o, lse, True, 1 / math.sqrt(D))
    A = torch.randn(2048, 4096, device="cuda", dtype=torch.bfloat16)
    W = torch.randn(4096, 4096, device="cuda", dtype=torch.bfloat16)
    for _ in range(2):
        ext.gemm(A, W, False, False)
    torch.cuda.synchronize()
    out.append({"small_cases": "ok", "attn_err": ext.attn_error_code(True), "gemm_err": ext.gemm_error_code(True)})
    print(json.dumps(out[-1]), flush=True)


def attn_large(ext, out):
    """One forward + backward at the Llama-3 8B shape (B1, S8192, H32/8, D128) for ncu."""
    B, S, H, Hk, D = 1, 8192, 32, 8, 128
    q = torch.randn(B, S, H, D, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(B, S, Hk, D, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(B, S, Hk, D, device="cuda", dtype=torch.bfloat16)
    o, lse = ext.attn_fwd(q, k, v, True, 1 / math.sqrt(D))
    ext.attn_bwd(torch.randn_like(o), q, k, v, o, lse, True, 1 / math.sqrt(D))
    torch.cuda.synchronize()
    out.append({"attn_large": "ok", "attn_err": ext.attn_error_code(True)})
    print(json.dumps(out[-1]), flush=True)


def mem_small(ext, out):
    """One launch each of the memory-bound kernels on >L2-sized inputs (for ncu)."""
    T, Dm, V = 8192, 4096, 32768
    x = torch.randn(T, Dm, device="cuda", dtype=torch.bfloat16)
    w = torch.ones(Dm, device="cuda", dtype=torch.bfloat16)
    y, rstd = ext.rmsnorm_fwd(x, w, 1e-5)
    ext.rmsnorm_bwd(x, x, w, rstd)
    a = torch.randn(T, 14336, device="cuda", dtype=torch.bfloat16)
    ext.swiglu_fwd(a, a)
    logits = torch.randn(T, V, device="cuda", dtype=torch.bfloat16)
    labels = torch.randint(0, V, (T,), device="cuda")
    loss, lse = ext.ce_fwd(logits, labels, -100)
    ext.ce_bwd(logits, labels, lse, torch.ones(1, device="cuda"), -100)
    n = 64 * 1024 * 1024
    p_, g_, m_, v_ = (torch.randn(n, device="cuda") for _ in range(4))
    ext.adamw([p_], [g_], [m_], [v_.abs()], 1e-3, 0.9, 0.95, 1e-8, 0.1, 1)
    torch.cuda.synchronize()
    out.append({"mem_small": "ok"})
    print(json.dumps(out[-1]), flush=True)


def bench_mxfp8(ext, out):
    """Block-scaled MXFP8 GEMM (codes + E8M0 scales already quantized) next to our bf16 GEMM
    and cuBLAS bf16 on the same shape, plus the quantizer's bandwidth."""
    from torchtitan_b200.ops.mx_gemm import mx_quantize

    for name, M, N, K in [("sq8192", 8192, 8192, 8192), ("w13_fwd", 8192, 28672, 4096), ("qkv_fwd", 8192, 6144, 4096)]:
        a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
        b = torch.randn(N, K, device="cuda", dtype=torch.bfloat16)
        qa, sa = mx_quantize(a)
        qb, sb = mx_quantize(b)
        mx = time_fn(lambda: ext.gemm_mxfp8(qa, sa, qb, sb))
        mx128 = time_fn(lambda: ext.gemm_mxfp8(qa, sa, qb, sb, 128))
        fa, ia = ext.f8_quantize(a, True)
        fb, ib = ext.f8_quantize(b, True)
        f8 = time_fn(lambda: ext.gemm_f8(fa, ia, fb, ib))
        f8q = time_fn(lambda: ext.f8_quantize(a, True))
        bf = time_fn(lambda: ext.gemm(a, b, False, False))
        lib = time_fn(lambda: torch.matmul(a, b.t()))
        q = time_fn(lambda: mx_quantize(a))
        fl = 2.0 * M * N * K
        out.append({"kernel": "gemm_mxfp8", "case": name, "M": M, "N": N, "K": K, "ms": mx, "tflops": fl / mx / 1e9,
                    "tile128_tflops": fl / mx128 / 1e9, "f8_rowwise_tflops": fl / f8 / 1e9,
                    "f8_quantize_gbs": a.numel() * 3 / f8q / 1e6, "bf16_tcgen05_tflops": fl / bf / 1e9, "cublas_bf16_tflops": fl / lib / 1e9,
                    "quantize_ms": q, "quantize_gbs": (a.numel() * 2 + a.numel() + a.numel() // 32) / q / 1e6,
                    "err": ext.mxgemm_error_code(True)})
        print(json.dumps(out[-1]), flush=True)


def bench_kda(ext, out):
    """Chunked KDA forward+backward (Kimi-Linear 48B layer shape: T 8192, 32 heads, K = V = 128)
    with the KDA kernels and with the PyTorch loops."""
    import os

    from torchtitan_b200.ops import kda

    B, T, H, K, V = 1, 8192, 32, 128, 128
    q, k = (torch.randn(B, T, H, K, device="cuda", requires_grad=True) for _ in range(2))
    v = torch.randn(B, T, H, V, device="cuda", requires_grad=True)
    g = (-torch.rand(B, T, H, K, device="cuda") * 0.1).requires_grad_()
    beta = torch.rand(B, T, H, device="cuda", requires_grad=True)
    do = torch.randn(B, T, H, V, device="cuda")

    def step():
        o, _ = kda.chunk_kda(q, k, v, g, beta)
        o.backward(do)

    res = {}
    for flag in ("1", "0"):
        os.environ["TTB_KDA_KERNEL"] = flag
        res[flag] = time_fn(step, iters=3, warmup=1, flush=False)
    os.environ.pop("TTB_KDA_KERNEL")
    out.append({"kernel": "kda_chunk", "case": f"B{B}_T{T}_H{H}_K{K}_V{V}", "fwd_bwd_ms_kernels": res["1"],
                "fwd_bwd_ms_torch": res["0"], "speedup": res["0"] / res["1"]})
    print(json.dumps(out[-1]), flush=True)


def bench_grouped_experts(ext, out):
    """Routed SwiGLU experts, forward + backward, on our grouped tcgen05 GEMMs against ATen's
    grouped GEMM (``torch._grouped_mm``, CUTLASS sm100) with the same SwiGLU. Shapes of the
    Kimi-Linear 48B layer per EP=8 rank: 32 local experts, hidden 2304, expert FFN 1024,
    65,536 routed rows (8,192 tokens x top-8) spread unevenly over the experts."""
    from torchtitan_b200.ops.moe import grouped_swiglu

    torch.manual_seed(0)
    E, D, H, rows = 32, 2304, 1024, 65536
    w = torch.rand(E, device="cuda") + 0.5
    counts = (w / w.sum() * rows).floor().long()
    counts[0] += rows - int(counts.sum())
    x = (torch.randn(rows, D, device="cuda") * 0.5).bfloat16().requires_grad_()
    w1, w3 = ((torch.randn(E, H, D, device="cuda") * 0.02).bfloat16().requires_grad_() for _ in range(2))
    w2 = (torch.randn(E, D, H, device="cuda") * 0.02).bfloat16().requires_grad_()
    dy = torch.randn(rows, D, device="cuda").bfloat16()
    offs = torch.cumsum(counts, 0).to(torch.int32)

    def ours():
        y = grouped_swiglu(x, w1, w2, w3, counts)
        y.backward(dy)

    def ours_mxfp8():
        from torchtitan_b200.ops.grouped import mx_grouped_swiglu_cuda

        y = mx_grouped_swiglu_cuda(x, w1, w2, w3, counts)
        y.backward(dy)

    def aten():
        h1 = torch._grouped_mm(x, w1.transpose(-2, -1), offs=offs)
        h3 = torch._grouped_mm(x, w3.transpose(-2, -1), offs=offs)
        a = torch.nn.functional.silu(h1) * h3
        y = torch._grouped_mm(a, w2.transpose(-2, -1), offs=offs)
        y.backward(dy)

    fl = 3 * 2 * 3 * rows * D * H  # three GEMMs, forward + two backward GEMMs each
    res = {"kernel": "grouped_swiglu_fwd_bwd", "E": E, "D": D, "H": H, "rows": rows}
    res["ours_ms"] = time_fn(ours)
    res["ours_tflops"] = fl / res["ours_ms"] / 1e9
    # MXFP8: forward and data-gradient GEMMs at FP8 rate (incl. quantization), weight grads bf16
    res["ours_mxfp8_ms"] = time_fn(ours_mxfp8)
    res["ours_mxfp8_tflops"] = fl / res["ours_mxfp8_ms"] / 1e9
    try:
        res["aten_grouped_mm_ms"] = time_fn(aten)
        res["aten_tflops"] = fl / res["aten_grouped_mm_ms"] / 1e9
    except Exception as e:  # noqa: BLE001 - record why the comparison is missing
        res["aten_error"] = repr(e)[:200]
    out.append(res)
    print(json.dumps(out[-1]), flush=True)


def bench_kda_vs_fla(ext, out):
    """Chunked KDA forward+backward against the fla library's ``chunk_kda`` (Triton, the
    reference's path: ``kimi_linear/model.py:559-571``) on the same inputs: H 32, K = V = 128,
    T 4096 and 131072; relative error of the outputs between the two."""
    from torchtitan_b200.ops import kda

    try:
        from fla.ops.kda import chunk_kda as fla_chunk_kda
    except Exception as e:  # noqa: BLE001
        out.append({"kernel": "kda_vs_fla", "unavailable": f"{type(e).__name__}: {e}"})
        print(json.dumps(out[-1]), flush=True)
        return
    for T in (4096, 131072):
        B, H, K, V = 1, 32, 128, 128
        torch.manual_seed(0)
        q, k = (torch.randn(B, T, H, K, device="cuda", dtype=torch.bfloat16, requires_grad=True) for _ in range(2))
        v = torch.randn(B, T, H, V, device="cuda", dtype=torch.bfloat16, requires_grad=True)
        g = (-torch.rand(B, T, H, K, device="cuda") * 0.1).requires_grad_()
        beta = torch.rand(B, T, H, device="cuda", requires_grad=True)
        do = torch.randn(B, T, H, V, device="cuda", dtype=torch.bfloat16)

        def ours():
            o, _ = kda.chunk_kda(q, k, v, g, beta, use_qk_l2norm=True)
            o.backward(do)
            return o

        def theirs():
            o, _ = fla_chunk_kda(q, k, v, g, beta, use_qk_l2norm_in_kernel=True)
            o.backward(do)
            return o

        with torch.no_grad():
            a = kda.chunk_kda(q, k, v, g, beta, use_qk_l2norm=True)[0].float()
            b = fla_chunk_kda(q, k, v, g, beta, use_qk_l2norm_in_kernel=True)[0].float()
        rel = float((a - b).norm() / b.norm())
        t_ours = time_fn(ours, iters=3, warmup=1, flush=False)
        t_fla = time_fn(theirs, iters=3, warmup=1, flush=False)
        out.append({"kernel": "kda_vs_fla", "case": f"B{B}_T{T}_H{H}_K{K}_V{V}", "fwd_bwd_ms_ours": t_ours,
                    "fwd_bwd_ms_fla": t_fla, "ours_over_fla_speed": t_fla / t_ours, "out_rel_err": rel})
        print(json.dumps(out[-1]), flush=True)
        del q, k, v, g, beta, do
        torch.cuda.empty_cache()


def bench_muon(ext, out):
    """Newton-Schulz (5 iterations) on a stack of 32 expert matrices of the Kimi-Linear 48B
    shape (1024 x 2304): batched through grouped GEMMs vs one matrix at a time."""
    from torchtitan_b200.components.optimizer import zeropower_via_newtonschulz5

    x = torch.randn(32, 1024, 2304, device="cuda")
    m, n = 1024, 2304
    flops = 32 * 5 * (2 * m * m * n * 2 + 2 * m * m * m)
    with torch.no_grad():
        t_b = time_fn(lambda: zeropower_via_newtonschulz5(x), iters=5, warmup=2, flush=False)
        t_l = time_fn(lambda: [zeropower_via_newtonschulz5(mm) for mm in x], iters=5, warmup=2, flush=False)
    out.append({"kernel": "muon_newton_schulz", "case": "32x1024x2304", "batched_ms": t_b, "loop_ms": t_l,
                "batched_tflops": flops / t_b / 1e9, "loop_tflops": flops / t_l / 1e9})
    print(json.dumps(out[-1]), flush=True)


def profile_case(ext, case: str) -> None:
    """Small fixed workloads for ncu captures of one kernel (``--only case:<name>``):
    gemm2 (bf16 4096^3), attn_fwd / attn_bwd (causal B1 S4096 H32/8 D128), kda (B1 T4096 H32
    K=V=128 forward+backward), adamw (4 x 64 Mi fp32 params, bf16 grads), rmsnorm (16384 x 4096
    forward and backward), grouped (routed SwiGLU experts forward+backward). Each runs the op a few
    times so ``-s`` can skip warm-up launches."""
    from torchtitan_b200 import ops

    torch.manual_seed(0)
    if case == "gemm2":
        a = torch.randn(4096, 4096, device="cuda").bfloat16()
        b = torch.randn(4096, 4096, device="cuda").bfloat16()
        for _ in range(3):
            ext.gemm(a, b, False, False)
    elif case in ("attn_fwd", "attn_bwd"):
        q = torch.randn(1, 4096, 32, 128, device="cuda", dtype=torch.bfloat16, requires_grad=True)
        k = torch.randn(1, 4096, 8, 128, device="cuda", dtype=torch.bfloat16, requires_grad=True)
        v = torch.randn(1, 4096, 8, 128, device="cuda", dtype=torch.bfloat16, requires_grad=True)
        for _ in range(3):
            o = ops.attention(q, k, v, causal=True)
            if case == "attn_bwd":
                o.backward(torch.randn_like(o))
    elif case == "kda":
        from torchtitan_b200.ops import kda

        q, k = (torch.randn(1, 4096, 32, 128, device="cuda", dtype=torch.bfloat16, requires_grad=True)
                for _ in range(2))
        v = torch.randn(1, 4096, 32, 128, device="cuda", dtype=torch.bfloat16, requires_grad=True)
        g = (-torch.rand(1, 4096, 32, 128, device="cuda") * 0.1).requires_grad_()
        beta = torch.rand(1, 4096, 32, device="cuda", requires_grad=True)
        for _ in range(2):
            o, _ = kda.chunk_kda(q, k, v, g, beta)
            o.backward(torch.randn_like(o))
    elif case == "grouped":
        # routed SwiGLU experts, Kimi-Linear 48B per-rank shape (32 experts, 2304 -> 1024, 65,536 rows)
        E, D, H, rows = 32, 2304, 1024, 65536
        w = torch.rand(E, device="cuda") + 0.5
        counts = (w / w.sum() * rows).floor().long()
        counts[0] += rows - int(counts.sum())
        x = (torch.randn(rows, D, device="cuda") * 0.5).bfloat16().requires_grad_()
        w1, w3 = ((torch.randn(E, H, D, device="cuda") * 0.02).bfloat16().requires_grad_() for _ in range(2))
        w2 = (torch.randn(E, D, H, device="cuda") * 0.02).bfloat16().requires_grad_()
        for _ in range(2):
            ops.grouped_swiglu(x, w1, w2, w3, counts).backward(torch.ones(rows, D, device="cuda").bfloat16())
    elif case == "rmsnorm":
        x = torch.randn(16384, 4096, device="cuda", dtype=torch.bfloat16)
        w = torch.ones(4096, device="cuda", dtype=torch.bfloat16)
        for _ in range(3):
            _, rstd = ext.rmsnorm_fwd(x, w, 1e-5)
            ext.rmsnorm_bwd(x, x, w, rstd)
    elif case == "adamw":
        n = 64 * 2 ** 20
        ps = [torch.randn(n, device="cuda") for _ in range(4)]
        gs = [torch.randn(n, device="cuda").bfloat16() for _ in range(4)]
        ms = [torch.zeros(n, device="cuda") for _ in range(4)]
        vs = [torch.zeros(n, device="cuda") for _ in range(4)]
        for s in range(1, 4):
            ops.fused_adamw_(ps, gs, ms, vs, lr=1e-3, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1, step=s)
    else:
        raise ValueError(f"unknown profile case {case}")
    torch.cuda.synchronize()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default="gemm,attn,mem")
    ap.add_argument("--out", default=None)
    a = ap.parse_args()
    from torchtitan_b200.ops._ext import ext as _e

    ext = _e()
    out: list = []
    sel = set(a.only.split(","))
    for item in sel:
        if item.startswith("case:"):
            profile_case(ext, item[5:])
    if "gemm" in sel:
        bench_gemm(ext, out)
    if "mxfp8" in sel:
        bench_mxfp8(ext, out)
    if "kda" in sel:
        bench_kda(ext, out)
    if "kda_fla" in sel:
        bench_kda_vs_fla(ext, out)
    if "grouped" in sel:
        bench_grouped_experts(ext, out)
    if "muon" in sel:
        bench_muon(ext, out)
    if "attn" in sel:
        bench_attn(ext, out)
    if "attn_large" in sel:
        attn_large(ext, out)
    if "mem_small" in sel:
        mem_small(ext, out)
    if "small" in sel:
        small_cases(ext, out)
    if "mem" in sel:
        bench_memory_bound(ext, out)
    if a.out:
        with open(a.out, "w") as f:
            for r in out:
                f.write(json.dumps(r) + "\n")


if __name__ == "__main__":
    main()
