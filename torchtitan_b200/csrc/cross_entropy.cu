// Cross entropy (sum over valid tokens) on bf16 logits without fp32 copies.
// Forward: one CTA per token row, single pass with an online (max, sum-exp)
// pair per thread, merged by shuffles; writes per-row loss and log-sum-exp,
// then a one-CTA deterministic sum.  Backward: one CTA per row writes
// (softmax - onehot) * g directly in bf16; g is read from device memory so no
// host synchronisation is needed.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "launch_api.h"

namespace ttb {
namespace {

using bf16 = __nv_bfloat16;
constexpr int NT = 512;

struct alignas(16) V8 {
  __nv_bfloat162 h[4];
};

__device__ __forceinline__ void merge(float& m, float& s, float m2, float s2) {
  const float mn = fmaxf(m, m2);
  if (mn == -INFINITY) return;
  s = s * __expf(m - mn) + s2 * __expf(m2 - mn);
  m = mn;
}

__device__ __forceinline__ float ex2f(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// Online (max, sum-exp) of 8 logits into a thread's running pair: the sum is kept relative to
// the running maximum and rescaled only when that maximum grows (one exponential per logit;
// exponentials as exp2 of x*log2(e) - m*log2(e), one FMA each).
__device__ __forceinline__ void accum8(const V8& v, float& m, float& s) {
  constexpr float kLog2e = 1.4426950408889634f;
  float f[8];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float2 t = __bfloat1622float2(v.h[j]);
    f[2 * j] = t.x;
    f[2 * j + 1] = t.y;
  }
  const float lm = fmaxf(fmaxf(fmaxf(f[0], f[1]), fmaxf(f[2], f[3])), fmaxf(fmaxf(f[4], f[5]), fmaxf(f[6], f[7])));
  if (lm > m) {
    s *= ex2f((m - lm) * kLog2e);  // m = -inf: s is 0 and stays 0
    m = lm;
  }
  const float mb = -m * kLog2e;
  float a = 0.f, b = 0.f;
#pragma unroll
  for (int j = 0; j < 8; j += 2) {
    a += ex2f(fmaf(f[j], kLog2e, mb));
    b += ex2f(fmaf(f[j + 1], kLog2e, mb));
  }
  s += a + b;
}

__global__ void __launch_bounds__(NT) ce_fwd_kernel(const bf16* __restrict__ logits, const int64_t* __restrict__ labels,
                                                    float* __restrict__ loss_rows, float* __restrict__ lse_out,
                                                    int64_t V, int64_t ignore_index) {
  const int64_t row = blockIdx.x;
  const bf16* x = logits + row * V;
  float m = -INFINITY, s = 0.f;
  const int64_t nv = V / 8;
  const V8* xv = reinterpret_cast<const V8*>(x);
  int64_t i = threadIdx.x;
  for (; i + NT < nv; i += 2 * NT) {  // two independent 16-byte loads in flight per thread
    const V8 v0 = xv[i], v1 = xv[i + NT];
    accum8(v0, m, s);
    accum8(v1, m, s);
  }
  if (i < nv) accum8(xv[i], m, s);
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    merge(m, s, m2, s2);
  }
  __shared__ float sm[NT / 32], ssum[NT / 32];
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  if (l == 0) {
    sm[w] = m;
    ssum[w] = s;
  }
  __syncthreads();
  if (w == 0) {
    m = l < NT / 32 ? sm[l] : -INFINITY;
    s = l < NT / 32 ? ssum[l] : 0.f;
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      merge(m, s, m2, s2);
    }
    if (l == 0) {
      const float lse = m + __logf(s);
      lse_out[row] = lse;
      const int64_t lab = labels[row];
      float loss = 0.f;
      if (lab != ignore_index && lab >= 0 && lab < V) loss = lse - __bfloat162float(x[lab]);
      loss_rows[row] = loss;
    }
  }
}

__global__ void sum_kernel(const float* __restrict__ v, float* __restrict__ out, int64_t n) {
  __shared__ double sh[1024 / 32];
  double acc = 0.0;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) acc += v[i];
#pragma unroll
  for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (threadIdx.x % 32 == 0) sh[threadIdx.x / 32] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    acc = threadIdx.x < blockDim.x / 32 ? sh[threadIdx.x] : 0.0;
#pragma unroll
    for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (threadIdx.x == 0) out[0] = static_cast<float>(acc);
  }
}

__global__ void __launch_bounds__(NT) ce_bwd_kernel(const bf16* __restrict__ logits, const int64_t* __restrict__ labels,
                                                    const float* __restrict__ lse, const float* __restrict__ gscale,
                                                    bf16* __restrict__ dlogits, int64_t V, int64_t ignore_index) {
  const int64_t row = blockIdx.x;
  const int64_t lab = labels[row];
  // rows the forward counts as loss 0 (ignore_index or a label outside [0, V)) get zero gradient
  const bool valid = lab != ignore_index && lab >= 0 && lab < V;
  const float g = valid ? gscale[0] : 0.f;
  const float L = lse[row];
  const bf16* x = logits + row * V;
  bf16* dx = dlogits + row * V;
  const int64_t nv = V / 8;
  for (int64_t i = threadIdx.x; i < nv; i += NT) {
    V8 v = reinterpret_cast<const V8*>(x)[i];
    V8 o;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 t = __bfloat1622float2(v.h[j]);
      const int64_t c = i * 8 + 2 * j;
      float a = __expf(t.x - L) - (c == lab ? 1.f : 0.f);
      float b = __expf(t.y - L) - (c + 1 == lab ? 1.f : 0.f);
      o.h[j] = __floats2bfloat162_rn(a * g, b * g);
    }
    reinterpret_cast<V8*>(dx)[i] = o;
  }
}

}  // namespace

void ce_fwd(const void* logits, const int64_t* labels, float* loss_rows, float* lse, float* loss_sum, int64_t T,
            int64_t V, int64_t ignore_index, cudaStream_t s) {
  if (V % 8) throw std::runtime_error("cross entropy: vocab must be a multiple of 8");
  if (T > 0)
    ce_fwd_kernel<<<static_cast<unsigned>(T), NT, 0, s>>>(static_cast<const bf16*>(logits), labels, loss_rows, lse, V,
                                                         ignore_index);
  sum_kernel<<<1, 1024, 0, s>>>(loss_rows, loss_sum, T);
  check_cuda(cudaGetLastError(), "ce_fwd");
}

void ce_bwd(const void* logits, const int64_t* labels, const float* lse, const float* gscale, void* dlogits, int64_t T,
            int64_t V, int64_t ignore_index, cudaStream_t s) {
  if (T == 0) return;
  ce_bwd_kernel<<<static_cast<unsigned>(T), NT, 0, s>>>(static_cast<const bf16*>(logits), labels, lse, gscale,
                                                       static_cast<bf16*>(dlogits), V, ignore_index);
  check_cuda(cudaGetLastError(), "ce_bwd");
}

}  // namespace ttb

// ---------------------------------------------------------------------------
// Allocation-free variant (declared in ce_noalloc.h): the per-row loss scratch
// is a fixed device array in this file instead of a buffer from the caller's
// allocator.
#include <atomic>
#include <cstdio>

#include "ce_noalloc.h"

namespace {

static __device__ __align__(256) float g_ce_rows_scratch[TTB_CE_NOALLOC_MAX_ROWS];

constexpr int kMaxDevices = 64;
// device address of the scratch array per device, resolved once; atomics make concurrent first
// calls from several host threads safe (both resolve the same address; either store wins)
std::atomic<float*> g_scratch_ptr[kMaxDevices] = {};
thread_local int g_last_cuda_error = 0;  // per host thread, so threads do not overwrite each other's code

}  // namespace

extern "C" int ttb_ce_fwd_noalloc_max_rows(void) { return TTB_CE_NOALLOC_MAX_ROWS; }

extern "C" int ttb_ce_fwd_noalloc_last_cuda_error(void) { return g_last_cuda_error; }

extern "C" int ttb_ce_fwd_noalloc(const void* logits, const int64_t* labels, int64_t T, int64_t V,
                                  int64_t ignore_index, float* lse, float* loss_sum, cudaStream_t stream) {
  if (T > TTB_CE_NOALLOC_MAX_ROWS) {
    std::fprintf(stderr, "ttb_ce_fwd_noalloc: %lld rows exceed the fixed scratch of %d rows\n",
                 static_cast<long long>(T), TTB_CE_NOALLOC_MAX_ROWS);
    return TTB_CE_NOALLOC_ETOOBIG;
  }
  if (T < 0 || V <= 0 || V % 8 || !lse || !loss_sum || (T > 0 && (!logits || !labels)))
    return TTB_CE_NOALLOC_EINVAL;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    g_last_cuda_error = static_cast<int>(e);
    return TTB_CE_NOALLOC_ECUDA;
  }
  float* rows = g_scratch_ptr[dev].load(std::memory_order_acquire);
  if (rows == nullptr) {
    // host code only knows a stand-in for the array; ask the runtime for its address on this device
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_ce_rows_scratch);
    if (e != cudaSuccess || p == nullptr) {
      g_last_cuda_error = static_cast<int>(e);
      return TTB_CE_NOALLOC_ECUDA;
    }
    rows = static_cast<float*>(p);
    g_scratch_ptr[dev].store(rows, std::memory_order_release);
  }
  if (T > 0)
    ttb::ce_fwd_kernel<<<static_cast<unsigned>(T), ttb::NT, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(logits), labels, rows, lse, V, ignore_index);
  ttb::sum_kernel<<<1, 1024, 0, stream>>>(rows, loss_sum, T);
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    g_last_cuda_error = static_cast<int>(e);
    return TTB_CE_NOALLOC_ECUDA;
  }
  return TTB_CE_NOALLOC_OK;
}
