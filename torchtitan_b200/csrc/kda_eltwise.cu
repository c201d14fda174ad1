// The element-wise pieces around KDA (Kimi Delta Attention), each one pass forward and
// one backward instead of a chain of PyTorch ops:
//   short conv   y[b,t,c] = silu(sum_{j<W} w[c,j] x[b, t-W+1+j, c])      (causal, depthwise)
//   gated norm   y[r,:]   = x[r,:] * rsqrt(mean(x[r,:]^2) + eps) * g * sigmoid(z[r,:])
//   decay gate   g[r,h,k] = -exp(A[h]) * softplus(x[r,h,k] + b[h,k])    (fp32 log decay)
// bf16 storage, fp32 arithmetic.  Weight gradients are accumulated per CTA in shared
// memory and added to an fp32 global buffer once per CTA.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <stdexcept>

#include "launch_api.h"

namespace ttb {
namespace kelt {

constexpr int NT = 256;
constexpr int MAXW = 8;

__device__ __forceinline__ float bf(const __nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float sigm(float x) { return 1.f / (1.f + __expf(-x)); }

// one thread per (b, t, c); grid-stride
__global__ void __launch_bounds__(NT) conv_fwd(const __nv_bfloat16* __restrict__ x, const float* __restrict__ w,
                                               __nv_bfloat16* __restrict__ y, int64_t B, int64_t T, int C, int W) {
  const int64_t n = B * T * C;
  for (int64_t i = blockIdx.x * (int64_t)NT + threadIdx.x; i < n; i += (int64_t)gridDim.x * NT) {
    const int c = static_cast<int>(i % C);
    const int64_t t = (i / C) % T;
    float a = 0.f;
    for (int j = 0; j < W; ++j) {
      const int64_t tt = t - W + 1 + j;
      if (tt >= 0) a += w[c * W + j] * bf(x[i + (tt - t) * C]);
    }
    y[i] = __float2bfloat16(a * sigm(a));
  }
}

// dx[b,t,c] = sum_j w[c,j] da[b, t+W-1-j, c];  dw[c,j] += sum_{b,t} da[b,t,c] x[b, t-W+1+j, c]
// with da = dy * silu'(a) recomputed.  Threads of a CTA own fixed channels c (grid over (C
// tiles, B*T tiles)), so dw accumulates in registers and is flushed once.
__global__ void __launch_bounds__(NT) conv_bwd(const __nv_bfloat16* __restrict__ x, const float* __restrict__ w,
                                               const __nv_bfloat16* __restrict__ dy, __nv_bfloat16* __restrict__ dx,
                                               float* __restrict__ dw, int64_t B, int64_t T, int C, int W,
                                               int rows_per_cta) {
  const int c = blockIdx.x * NT + threadIdx.x;
  if (c >= C) return;
  const int64_t r0 = static_cast<int64_t>(blockIdx.y) * rows_per_cta;  // rows = (b, t) pairs
  const int64_t r1 = min(r0 + rows_per_cta, B * T);
  float wc[MAXW], dwc[MAXW];
  for (int j = 0; j < W; ++j) {
    wc[j] = w[c * W + j];
    dwc[j] = 0.f;
  }
  for (int64_t r = r0; r < r1; ++r) {
    const int64_t t = r % T;
    // da at row r
    {
      float a = 0.f;
      for (int j = 0; j < W; ++j) {
        const int64_t tt = t - W + 1 + j;
        if (tt >= 0) a += wc[j] * bf(x[(r + tt - t) * C + c]);
      }
      const float s = sigm(a);
      const float da = bf(dy[r * C + c]) * s * (1.f + a * (1.f - s));
      for (int j = 0; j < W; ++j) {
        const int64_t tt = t - W + 1 + j;
        if (tt >= 0) dwc[j] += da * bf(x[(r + tt - t) * C + c]);
      }
    }
    // dx at row r: needs da at rows t .. t+W-1 (same sequence)
    float g = 0.f;
    for (int j = 0; j < W; ++j) {
      const int64_t to = t + W - 1 - j;  // output position that reads x[t] with tap j
      if (to >= T) continue;
      const int64_t ro = r + (to - t);
      float a = 0.f;
      for (int q = 0; q < W; ++q) {
        const int64_t tt = to - W + 1 + q;
        if (tt >= 0) a += wc[q] * bf(x[(ro + tt - to) * C + c]);
      }
      const float s = sigm(a);
      g += wc[j] * bf(dy[ro * C + c]) * s * (1.f + a * (1.f - s));
    }
    dx[r * C + c] = __float2bfloat16(g);
  }
  for (int j = 0; j < W; ++j) atomicAdd(dw + c * W + j, dwc[j]);
}

// one CTA per row
__global__ void __launch_bounds__(NT) gnorm_fwd(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ z,
                                                const float* __restrict__ g, __nv_bfloat16* __restrict__ y, int D,
                                                float eps) {
  __shared__ float red[NT / 32];
  const size_t off = static_cast<size_t>(blockIdx.x) * D;
  float ss = 0.f;
  for (int d = threadIdx.x; d < D; d += NT) {
    const float v = bf(x[off + d]);
    ss += v * v;
  }
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < NT / 32; ++i) tot += red[i];
  const float r = rsqrtf(tot / D + eps);
  for (int d = threadIdx.x; d < D; d += NT)
    y[off + d] = __float2bfloat16(bf(x[off + d]) * r * g[d] * sigm(bf(z[off + d])));
}

// dy -> dx, dz (per row) and dg (summed over rows: per-CTA shared accumulators, one atomic flush)
__global__ void __launch_bounds__(NT) gnorm_bwd(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ z,
                                                const float* __restrict__ g, const __nv_bfloat16* __restrict__ dy,
                                                __nv_bfloat16* __restrict__ dx, __nv_bfloat16* __restrict__ dz,
                                                float* __restrict__ dg, int64_t R, int D, float eps) {
  extern __shared__ float sdg[];  // [D]
  __shared__ float red[2][NT / 32];
  for (int d = threadIdx.x; d < D; d += NT) sdg[d] = 0.f;
  for (int64_t row = blockIdx.x; row < R; row += gridDim.x) {
    const size_t off = static_cast<size_t>(row) * D;
    float ss = 0.f, dot = 0.f;  // sum x^2, sum x * (dy g sigma(z))
    for (int d = threadIdx.x; d < D; d += NT) {
      const float v = bf(x[off + d]);
      ss += v * v;
      dot += v * bf(dy[off + d]) * g[d] * sigm(bf(z[off + d]));
    }
    for (int o = 16; o > 0; o >>= 1) {
      ss += __shfl_xor_sync(0xffffffffu, ss, o);
      dot += __shfl_xor_sync(0xffffffffu, dot, o);
    }
    if (threadIdx.x % 32 == 0) {
      red[0][threadIdx.x / 32] = ss;
      red[1][threadIdx.x / 32] = dot;
    }
    __syncthreads();
    float tss = 0.f, tdot = 0.f;
    for (int i = 0; i < NT / 32; ++i) {
      tss += red[0][i];
      tdot += red[1][i];
    }
    __syncthreads();
    const float r = rsqrtf(tss / D + eps);
    for (int d = threadIdx.x; d < D; d += NT) {
      const float v = bf(x[off + d]), zz = bf(z[off + d]), s = sigm(zz), gy = bf(dy[off + d]);
      const float n = v * r;  // normalised x
      dz[off + d] = __float2bfloat16(gy * n * g[d] * s * (1.f - s));
      sdg[d] += gy * n * s;
      // y = n g s; dx = r (h - n mean(n h)) with h = dy g s
      dx[off + d] = __float2bfloat16(r * (gy * g[d] * s - n * r * tdot / D));
    }
  }
  __syncthreads();
  for (int d = threadIdx.x; d < D; d += NT) atomicAdd(dg + d, sdg[d]);
}

// one thread per element; the per-(h, k) parameter gradients accumulate per CTA in shared memory
__global__ void __launch_bounds__(NT) gate_fwd(const __nv_bfloat16* __restrict__ x, const float* __restrict__ A,
                                               const float* __restrict__ b, float* __restrict__ g, int64_t n, int H,
                                               int K) {
  for (int64_t i = blockIdx.x * (int64_t)NT + threadIdx.x; i < n; i += (int64_t)gridDim.x * NT) {
    const int hk = static_cast<int>(i % (H * K));
    const float v = bf(x[i]) + (b != nullptr ? b[hk] : 0.f);
    const float sp = v > 20.f ? v : log1pf(__expf(v));
    g[i] = -__expf(A[hk / K]) * sp;
  }
}

__global__ void __launch_bounds__(NT) gate_bwd(const __nv_bfloat16* __restrict__ x, const float* __restrict__ A,
                                               const float* __restrict__ b, const float* __restrict__ dg,
                                               __nv_bfloat16* __restrict__ dx, float* __restrict__ dA,
                                               float* __restrict__ db, int64_t n, int H, int K) {
  extern __shared__ float acc[];  // [H*K] db partials, then [H] dA partials
  for (int j = threadIdx.x; j < H * K + H; j += NT) acc[j] = 0.f;
  __syncthreads();
  for (int64_t i = blockIdx.x * (int64_t)NT + threadIdx.x; i < n; i += (int64_t)gridDim.x * NT) {
    const int hk = static_cast<int>(i % (H * K));
    const float v = bf(x[i]) + (b != nullptr ? b[hk] : 0.f);
    const float sp = v > 20.f ? v : log1pf(__expf(v));
    const float e = __expf(A[hk / K]);
    const float d = dg[i];
    const float dv = -d * e * sigm(v);
    dx[i] = __float2bfloat16(dv);
    atomicAdd(acc + hk, dv);
    atomicAdd(acc + H * K + hk / K, -d * e * sp);
  }
  __syncthreads();
  for (int j = threadIdx.x; j < H * K; j += NT)
    if (db != nullptr) atomicAdd(db + j, acc[j]);
  for (int j = threadIdx.x; j < H; j += NT) atomicAdd(dA + j, acc[H * K + j]);
}

int sms() {
  int dev = 0, n = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

}  // namespace kelt

void kda_short_conv_fwd(const void* x, const float* w, void* y, int64_t B, int64_t T, int C, int W, cudaStream_t s) {
  using namespace kelt;
  if (W < 1 || W > MAXW) throw std::runtime_error("short conv: kernel width 1..8");
  const int64_t n = B * T * C;
  if (n == 0) return;
  const int64_t blocks = (n + NT - 1) / NT;
  conv_fwd<<<(unsigned)(blocks < 16 * sms() ? blocks : 16 * sms()), NT, 0, s>>>(
      static_cast<const __nv_bfloat16*>(x), w, static_cast<__nv_bfloat16*>(y), B, T, C, W);
  check_cuda(cudaGetLastError(), "short conv fwd launch");
}

void kda_short_conv_bwd(const void* x, const float* w, const void* dy, void* dx, float* dw, int64_t B, int64_t T,
                        int C, int W, cudaStream_t s) {
  using namespace kelt;
  if (W < 1 || W > MAXW) throw std::runtime_error("short conv: kernel width 1..8");
  check_cuda(cudaMemsetAsync(dw, 0, sizeof(float) * C * W, s), "short conv dw clear");
  const int64_t rows = B * T;
  if (rows == 0) return;
  const int ctiles = (C + NT - 1) / NT;
  const int64_t want = 8LL * sms();
  int64_t rtiles = (want + ctiles - 1) / ctiles;
  rtiles = rtiles < rows ? rtiles : rows;
  const int rows_per = static_cast<int>((rows + rtiles - 1) / rtiles);
  rtiles = (rows + rows_per - 1) / rows_per;
  conv_bwd<<<dim3(ctiles, (unsigned)rtiles), NT, 0, s>>>(
      static_cast<const __nv_bfloat16*>(x), w, static_cast<const __nv_bfloat16*>(dy), static_cast<__nv_bfloat16*>(dx),
      dw, B, T, C, W, rows_per);
  check_cuda(cudaGetLastError(), "short conv bwd launch");
}

void kda_gated_norm_fwd(const void* x, const void* z, const float* g, void* y, int64_t R, int D, float eps,
                        cudaStream_t s) {
  using namespace kelt;
  if (R == 0) return;
  if (R > 0x7fffffff) throw std::runtime_error("gated norm: too many rows");
  kelt::gnorm_fwd<<<(unsigned)R, NT, 0, s>>>(static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(z),
                                             g, static_cast<__nv_bfloat16*>(y), D, eps);
  check_cuda(cudaGetLastError(), "gated norm fwd launch");
}

void kda_gated_norm_bwd(const void* x, const void* z, const float* g, const void* dy, void* dx, void* dz, float* dg,
                        int64_t R, int D, float eps, cudaStream_t s) {
  using namespace kelt;
  const size_t sm = sizeof(float) * D;
  if (sm > 200 * 1024) throw std::runtime_error("gated norm: width too large");
  check_cuda(cudaMemsetAsync(dg, 0, sm, s), "gated norm dg clear");
  if (R == 0) return;
  check_cuda(cudaFuncSetAttribute(gnorm_bwd, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm), "gated norm smem");
  const int64_t grid = R < 4LL * sms() ? R : 4LL * sms();
  gnorm_bwd<<<(unsigned)grid, NT, sm, s>>>(static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(z),
                                           g, static_cast<const __nv_bfloat16*>(dy), static_cast<__nv_bfloat16*>(dx),
                                           static_cast<__nv_bfloat16*>(dz), dg, R, D, eps);
  check_cuda(cudaGetLastError(), "gated norm bwd launch");
}

void kda_gate_fwd(const void* x, const float* A, const float* b, float* g, int64_t n, int H, int K, cudaStream_t s) {
  using namespace kelt;
  if (n == 0) return;
  const int64_t blocks = (n + NT - 1) / NT;
  gate_fwd<<<(unsigned)(blocks < 16 * sms() ? blocks : 16 * sms()), NT, 0, s>>>(static_cast<const __nv_bfloat16*>(x),
                                                                                A, b, g, n, H, K);
  check_cuda(cudaGetLastError(), "kda gate fwd launch");
}

void kda_gate_bwd(const void* x, const float* A, const float* b, const float* dg, void* dx, float* dA, float* db,
                  int64_t n, int H, int K, cudaStream_t s) {
  using namespace kelt;
  const size_t sm = sizeof(float) * (static_cast<size_t>(H) * K + H);
  if (sm > 200 * 1024) throw std::runtime_error("kda gate: too many channels");
  check_cuda(cudaMemsetAsync(dA, 0, sizeof(float) * H, s), "kda gate dA clear");
  if (db != nullptr) check_cuda(cudaMemsetAsync(db, 0, sizeof(float) * H * K, s), "kda gate db clear");
  if (n == 0) return;
  check_cuda(cudaFuncSetAttribute(gate_bwd, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm), "kda gate smem");
  const int64_t blocks = (n + NT - 1) / NT;
  gate_bwd<<<(unsigned)(blocks < 4 * sms() ? blocks : 4 * sms()), NT, sm, s>>>(
      static_cast<const __nv_bfloat16*>(x), A, b, dg, static_cast<__nv_bfloat16*>(dx), dA, db, n, H, K);
  check_cuda(cudaGetLastError(), "kda gate bwd launch");
}

}  // namespace ttb
