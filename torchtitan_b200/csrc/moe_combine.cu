// Deterministic MoE combine (token un-permute + gate-weighted sum) and its backward.
//
// The routed rows y [R, D] (bf16) are sorted by expert; pos[t, j] is the sorted row that holds
// slot j of token t.  Forward, per token (no atomics, fixed summation order):
//     out[t] = base[t] + sum_j w[t, j] * y[pos[t, j]]        (fp32 accumulation, one bf16 rounding)
// with base optional (shared experts' output) and w optional (gates already applied before the
// experts).  Backward:
//     dy[r]   = w_sorted[r] * dout[token_of[r]]             (a gather: every sorted row is one slot)
//     dw[t,j] = dot(dout[t], y[pos[t, j]])                   (fp32, one warp per slot)
// Rows are 16-byte vectors of 8 bf16; D must be a multiple of 8.  Indices outside [0, rows) read
// as zero rows and are never written through.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <stdexcept>

#include "launch_api.h"

namespace ttb {
namespace {

using bf16 = __nv_bfloat16;

struct alignas(16) V8 {
  __nv_bfloat162 h[4];
};

__device__ __forceinline__ void add8(float (&acc)[8], const V8& v, float w) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(v.h[i]);
    acc[2 * i] = fmaf(w, f.x, acc[2 * i]);
    acc[2 * i + 1] = fmaf(w, f.y, acc[2 * i + 1]);
  }
}

__device__ __forceinline__ V8 pack8(const float (&acc)[8]) {
  V8 o;
#pragma unroll
  for (int i = 0; i < 4; ++i) o.h[i] = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
  return o;
}

// one warp per token; lanes stride over the row's 16-byte vectors
__global__ void __launch_bounds__(256) combine_fwd_kernel(const bf16* __restrict__ base, const bf16* __restrict__ y,
                                                          const int64_t* __restrict__ pos, const float* __restrict__ w,
                                                          bf16* __restrict__ out, int64_t T, int k, int d8,
                                                          int64_t R) {
  const int64_t t = static_cast<int64_t>(blockIdx.x) * 8 + threadIdx.x / 32;
  if (t >= T) return;
  const int lane = threadIdx.x % 32;
  const V8* yv = reinterpret_cast<const V8*>(y);
  for (int c = lane; c < d8; c += 32) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (base) add8(acc, reinterpret_cast<const V8*>(base)[t * d8 + c], 1.f);
    for (int j = 0; j < k; ++j) {
      const int64_t r = pos[t * k + j];
      if (r < 0 || r >= R) continue;
      add8(acc, yv[r * d8 + c], w ? w[t * k + j] : 1.f);
    }
    reinterpret_cast<V8*>(out)[t * d8 + c] = pack8(acc);
  }
}

// dy[r] = scale[r] * dout[token_of[r]]; one warp per sorted row
__global__ void __launch_bounds__(256) combine_bwd_rows_kernel(const bf16* __restrict__ dout,
                                                               const int64_t* __restrict__ token_of,
                                                               const float* __restrict__ scale, bf16* __restrict__ dy,
                                                               int64_t R, int d8, int64_t T) {
  const int64_t r = static_cast<int64_t>(blockIdx.x) * 8 + threadIdx.x / 32;
  if (r >= R) return;
  const int lane = threadIdx.x % 32;
  const int64_t t = token_of[r];
  const bool live = t >= 0 && t < T;
  const float s = scale ? scale[r] : 1.f;
  for (int c = lane; c < d8; c += 32) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (live) add8(acc, reinterpret_cast<const V8*>(dout)[t * d8 + c], s);
    reinterpret_cast<V8*>(dy)[r * d8 + c] = pack8(acc);
  }
}

// dw[t, j] = dot(dout[t], y[pos[t, j]]); one warp per slot, lanes reduce by shuffles
__global__ void __launch_bounds__(256) combine_bwd_gates_kernel(const bf16* __restrict__ dout,
                                                                const bf16* __restrict__ y,
                                                                const int64_t* __restrict__ pos,
                                                                float* __restrict__ dw, int64_t slots, int k, int d8,
                                                                int64_t R) {
  const int64_t s = static_cast<int64_t>(blockIdx.x) * 8 + threadIdx.x / 32;
  if (s >= slots) return;
  const int lane = threadIdx.x % 32;
  const int64_t t = s / k, r = pos[s];
  float acc = 0.f;
  if (r >= 0 && r < R) {
    const V8* a = reinterpret_cast<const V8*>(dout) + t * d8;
    const V8* b = reinterpret_cast<const V8*>(y) + r * d8;
    for (int c = lane; c < d8; c += 32) {
      const V8 va = a[c], vb = b[c];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 fa = __bfloat1622float2(va.h[i]), fb = __bfloat1622float2(vb.h[i]);
        acc = fmaf(fa.x, fb.x, acc);
        acc = fmaf(fa.y, fb.y, acc);
      }
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) dw[s] = acc;
}

}  // namespace

void moe_combine_fwd(const void* base, const void* y, const int64_t* pos, const float* w, void* out, int64_t T,
                     int k, int64_t D, int64_t R, cudaStream_t s) {
  if (D % 8) throw std::runtime_error("moe_combine: row length must be a multiple of 8");
  if (T == 0) return;
  combine_fwd_kernel<<<static_cast<unsigned>((T + 7) / 8), 256, 0, s>>>(
      static_cast<const bf16*>(base), static_cast<const bf16*>(y), pos, w, static_cast<bf16*>(out), T, k,
      static_cast<int>(D / 8), R);
  check_cuda(cudaGetLastError(), "moe_combine_fwd");
}

void moe_combine_bwd(const void* dout, const void* y, const int64_t* pos, const int64_t* token_of,
                     const float* scale, void* dy, float* dw, int64_t T, int k, int64_t D, int64_t R,
                     cudaStream_t s) {
  if (D % 8) throw std::runtime_error("moe_combine: row length must be a multiple of 8");
  if (R > 0)
    combine_bwd_rows_kernel<<<static_cast<unsigned>((R + 7) / 8), 256, 0, s>>>(
        static_cast<const bf16*>(dout), token_of, scale, static_cast<bf16*>(dy), R, static_cast<int>(D / 8), T);
  if (dw != nullptr && T * k > 0)
    combine_bwd_gates_kernel<<<static_cast<unsigned>((T * k + 7) / 8), 256, 0, s>>>(
        static_cast<const bf16*>(dout), static_cast<const bf16*>(y), pos, dw, T * k, k, static_cast<int>(D / 8), R);
  check_cuda(cudaGetLastError(), "moe_combine_bwd");
}

}  // namespace ttb
