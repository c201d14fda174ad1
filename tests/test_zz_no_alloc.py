"""The allocation-free cross-entropy forward, called through its exported C symbol.

It serves callers that cannot allocate device memory (allocator callbacks,
pre-reserved devices, C-only runtimes); it must give the same loss and
log-sum-exp as the regular extension entry point.  Two calls in a row check
that the shared scratch array left by one call does not leak into the next.
This file sorts last so a fail-fast run has already run every other test.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    import torchtitan_b200._C as c  # noqa: F401  (loads the library and its torch deps)

    lib = ctypes.CDLL(c.__file__)
    f = lib.ttb_ce_fwd_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                  ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    lib.ttb_ce_fwd_noalloc_max_rows.restype = ctypes.c_int
    return lib


def _call(lib, logits, labels, lse, loss):
    stream = torch.cuda.current_stream().cuda_stream
    return lib.ttb_ce_fwd_noalloc(logits.data_ptr(), labels.data_ptr(), logits.shape[0], logits.shape[1], -100,
                                  lse.data_ptr(), loss.data_ptr(), stream)


def test_no_alloc_matches_regular_entry_point():
    from torchtitan_b200.ops._ext import ext

    lib = _lib()
    torch.manual_seed(11)
    # second call has fewer rows than the first: stale scratch rows must not be summed
    for T, V in [(513, 2048), (257, 128256)]:
        logits = (3 * torch.randn(T, V, device="cuda")).to(torch.bfloat16)
        labels = torch.randint(0, V, (T,), device="cuda")
        labels[::5] = -100
        lse = torch.empty(T, device="cuda")
        loss = torch.empty(1, device="cuda")
        assert _call(lib, logits, labels, lse, loss) == 0
        ref_loss, ref_lse = ext().ce_fwd(logits, labels, -100)
        torch.cuda.synchronize()
        assert abs(loss.item() - ref_loss.item()) <= 1e-3 * abs(ref_loss.item())
        assert ((lse - ref_lse).norm() / ref_lse.norm()).item() < 1e-5
        # and against plain fp32 PyTorch on the same bf16 logits
        x32 = logits.float()
        f32_loss = torch.nn.functional.cross_entropy(x32, labels, ignore_index=-100, reduction="sum")
        f32_lse = torch.logsumexp(x32, dim=-1)
        assert abs(loss.item() - f32_loss.item()) <= 1e-3 * abs(f32_loss.item())
        assert ((lse - f32_lse).norm() / f32_lse.norm()).item() < 1e-5


def test_no_alloc_rejects_oversize():
    lib = _lib()
    big = lib.ttb_ce_fwd_noalloc_max_rows() + 1
    logits = torch.empty(1, 8, device="cuda", dtype=torch.bfloat16)
    labels = torch.zeros(1, device="cuda", dtype=torch.int64)
    out = torch.empty(1, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.ttb_ce_fwd_noalloc(logits.data_ptr(), labels.data_ptr(), big, 8, -100, out.data_ptr(), out.data_ptr(),
                                stream)
    assert rc == 1
