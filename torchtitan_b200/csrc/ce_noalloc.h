// Allocation-free cross-entropy forward, callable from C.
//
// This entry point has no counterpart in the reference (which has no native
// code at all).  It exists for callers that cannot allocate GPU memory
// themselves: code running inside a custom allocator or memory-pool callback,
// a host that has reserved the whole device up front and hands out fixed
// buffers, or a runtime whose only interface to this library is a C symbol
// (no PyTorch, hence no caching allocator).  Such callers pass inputs and
// outputs; the per-row loss scratch this kernel needs lives in a fixed device
// array inside the library instead of being allocated per call.
//
// Limits and sharing rules:
//   * at most TTB_CE_NOALLOC_MAX_ROWS token rows per call (65536 rows, 256 KiB
//     of device memory held by every GPU that loads the library until exit);
//     larger T is rejected with TTB_CE_NOALLOC_ETOOBIG and nothing is launched;
//   * all calls in the process share that one scratch array, so two calls that
//     overlap on the GPU (different streams, or different host threads using
//     the same device) race and give wrong results; serialise them;
//   * the scratch keeps the previous call's contents; nothing needs to start
//     at zero because every row of the current call is written before it is read;
//   * labels outside [0, V) that are not ignore_index count as ignored rows (loss 0),
//     unlike torch.nn.functional.cross_entropy, which rejects them; validate labels first
//     if that matters;
//   * host-thread safety: the per-device address cache is atomic and the last CUDA error
//     code is kept per host thread, so concurrent calls are safe on the host side (they
//     still race on the GPU, see above);
//   * the first call on each device resolves the scratch array's device address
//     (cudaGetSymbolAddress with that device current); make that first call
//     before any stream capture.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TTB_CE_NOALLOC_MAX_ROWS 65536
#define TTB_CE_NOALLOC_OK 0
#define TTB_CE_NOALLOC_ETOOBIG 1   // T > TTB_CE_NOALLOC_MAX_ROWS
#define TTB_CE_NOALLOC_EINVAL 2    // T < 0, V not a positive multiple of 8, or a null pointer
#define TTB_CE_NOALLOC_ECUDA 3     // a CUDA call failed (see ttb_ce_fwd_noalloc_last_cuda_error)

// logits: bf16 [T, V] row-major on the current device; labels: int64 [T]
// (ignore_index rows contribute 0).  Outputs: lse fp32 [T] (natural-log
// log-sum-exp per row) and loss_sum fp32 [1] (sum of per-row losses).
// Work is enqueued on `stream`; the function does not synchronise.
int ttb_ce_fwd_noalloc(const void* logits, const int64_t* labels, int64_t T, int64_t V, int64_t ignore_index,
                       float* lse, float* loss_sum, cudaStream_t stream);

int ttb_ce_fwd_noalloc_max_rows(void);
int ttb_ce_fwd_noalloc_last_cuda_error(void);  // of the calling host thread

#ifdef __cplusplus
}
#endif
