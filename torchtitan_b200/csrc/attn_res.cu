// Block Attention-Residual mixing in one pass per token (forward and backward).
//
// For one token with block vectors V_0..V_N (the completed blocks and the partial sum,
// each of width D), norm weight g and pseudo-query w (u = g * w elementwise):
//   r_n = 1 / sqrt(mean(V_n^2) + eps),  l_n = r_n (V_n . u),  p = softmax(l),  O = sum_n p_n V_n
// Backward with dO:
//   dp_n = dO . V_n,  dl_n = p_n (dp_n - sum_m p_m dp_m)
//   dV_n = p_n dO + dl_n r_n (u - r_n^2 (V_n . u) / D * V_n)
//   du  += sum_n dl_n r_n V_n        (summed over tokens; dw = du * g, dg = du * w on the host)
// The block vectors are read in place (no stacked copy).  A CTA walks tokens with a grid
// stride: pass 1 forms the per-block dot products (block-wide reductions), pass 2 writes
// the outputs.  bf16 storage, fp32 arithmetic.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <stdexcept>

#include "launch_api.h"

namespace ttb {
namespace attnres_impl {

constexpr int MAXB = 17;  // completed blocks + the partial one
constexpr int NT = 256;
constexpr int NW = NT / 32;

struct Blocks {
  const __nv_bfloat16* v[MAXB];
  __nv_bfloat16* dv[MAXB];
  int n;
};

// sums vals[0..n) over the CTA; every thread gets the totals in vals
template <int CAP>
__device__ void block_sum(float* vals, int n, float (*red)[NW]) {
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  for (int i = 0; i < n; ++i) {
    float v = vals[i];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    if (lane == 0) red[i][warp] = v;
  }
  __syncthreads();
  for (int i = 0; i < n; ++i) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) s += red[i][w];
    vals[i] = s;
  }
  __syncthreads();
}

__global__ void __launch_bounds__(NT) fwd_kernel(Blocks b, const float* __restrict__ u, __nv_bfloat16* __restrict__ out,
                                                 int64_t T, int D, float eps) {
  __shared__ float red[2 * MAXB][NW];
  for (int64_t t = blockIdx.x; t < T; t += gridDim.x) {
    float acc[2 * MAXB];
    for (int n = 0; n < b.n; ++n) acc[2 * n] = acc[2 * n + 1] = 0.f;
    for (int d = threadIdx.x; d < D; d += NT) {
      const float ud = u[d];
      for (int n = 0; n < b.n; ++n) {
        const float x = __bfloat162float(b.v[n][t * D + d]);
        acc[2 * n] += x * x;
        acc[2 * n + 1] += x * ud;
      }
    }
    block_sum<2 * MAXB>(acc, 2 * b.n, red);
    float p[MAXB], mx = -INFINITY;
    for (int n = 0; n < b.n; ++n) {
      p[n] = rsqrtf(acc[2 * n] / D + eps) * acc[2 * n + 1];
      mx = fmaxf(mx, p[n]);
    }
    float z = 0.f;
    for (int n = 0; n < b.n; ++n) {
      p[n] = __expf(p[n] - mx);
      z += p[n];
    }
    for (int n = 0; n < b.n; ++n) p[n] /= z;
    for (int d = threadIdx.x; d < D; d += NT) {
      float o = 0.f;
      for (int n = 0; n < b.n; ++n) o += p[n] * __bfloat162float(b.v[n][t * D + d]);
      out[t * D + d] = __float2bfloat16(o);
    }
  }
}

__global__ void __launch_bounds__(NT) bwd_kernel(Blocks b, const float* __restrict__ u,
                                                 const __nv_bfloat16* __restrict__ dout, float* __restrict__ du,
                                                 int64_t T, int D, float eps) {
  __shared__ float red[3 * MAXB][NW];
  extern __shared__ float du_acc[];  // [D] this CTA's share of du
  for (int d = threadIdx.x; d < D; d += NT) du_acc[d] = 0.f;
  for (int64_t t = blockIdx.x; t < T; t += gridDim.x) {
    float acc[3 * MAXB];
    for (int n = 0; n < b.n; ++n) acc[3 * n] = acc[3 * n + 1] = acc[3 * n + 2] = 0.f;
    for (int d = threadIdx.x; d < D; d += NT) {
      const float ud = u[d], g = __bfloat162float(dout[t * D + d]);
      for (int n = 0; n < b.n; ++n) {
        const float x = __bfloat162float(b.v[n][t * D + d]);
        acc[3 * n] += x * x;
        acc[3 * n + 1] += x * ud;
        acc[3 * n + 2] += x * g;
      }
    }
    block_sum<3 * MAXB>(acc, 3 * b.n, red);
    float p[MAXB], r[MAXB], mx = -INFINITY;
    for (int n = 0; n < b.n; ++n) {
      r[n] = rsqrtf(acc[3 * n] / D + eps);
      p[n] = r[n] * acc[3 * n + 1];
      mx = fmaxf(mx, p[n]);
    }
    float z = 0.f;
    for (int n = 0; n < b.n; ++n) {
      p[n] = __expf(p[n] - mx);
      z += p[n];
    }
    float pdp = 0.f;
    for (int n = 0; n < b.n; ++n) {
      p[n] /= z;
      pdp += p[n] * acc[3 * n + 2];
    }
    float dl[MAXB], cu[MAXB], cv[MAXB];
    for (int n = 0; n < b.n; ++n) {
      dl[n] = p[n] * (acc[3 * n + 2] - pdp);
      cu[n] = dl[n] * r[n];                                    // coefficient of u in dV_n, and of V_n in du
      cv[n] = -dl[n] * r[n] * r[n] * r[n] * acc[3 * n + 1] / D;  // coefficient of V_n in dV_n
    }
    for (int d = threadIdx.x; d < D; d += NT) {
      const float ud = u[d], g = __bfloat162float(dout[t * D + d]);
      float dua = 0.f;
      for (int n = 0; n < b.n; ++n) {
        const float x = __bfloat162float(b.v[n][t * D + d]);
        b.dv[n][t * D + d] = __float2bfloat16(p[n] * g + cu[n] * ud + cv[n] * x);
        dua += cu[n] * x;
      }
      du_acc[d] += dua;
    }
  }
  __syncthreads();
  for (int d = threadIdx.x; d < D; d += NT) atomicAdd(du + d, du_acc[d]);
}

int grid_for(int64_t T) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t g = static_cast<int64_t>(sms) * 4;
  return static_cast<int>(T < g ? T : g);
}

}  // namespace attnres_impl

void attn_res_fwd(const void* const* blocks, int nb, const float* u, void* out, int64_t T, int D, float eps,
                  cudaStream_t s) {
  using namespace attnres_impl;
  if (nb < 1 || nb > MAXB) throw std::runtime_error("attn_res: 1..17 blocks");
  if (T == 0) return;
  Blocks b{};
  b.n = nb;
  for (int i = 0; i < nb; ++i) b.v[i] = static_cast<const __nv_bfloat16*>(blocks[i]);
  fwd_kernel<<<grid_for(T), NT, 0, s>>>(b, u, static_cast<__nv_bfloat16*>(out), T, D, eps);
  check_cuda(cudaGetLastError(), "attn_res fwd launch");
}

void attn_res_bwd(const void* const* blocks, void* const* dblocks, int nb, const float* u, const void* dout, float* du,
                  int64_t T, int D, float eps, cudaStream_t s) {
  using namespace attnres_impl;
  if (nb < 1 || nb > MAXB) throw std::runtime_error("attn_res: 1..17 blocks");
  const size_t sm = static_cast<size_t>(D) * sizeof(float);
  if (sm > 200 * 1024) throw std::runtime_error("attn_res: width too large");
  check_cuda(cudaMemsetAsync(du, 0, sm, s), "attn_res du clear");
  if (T == 0) return;
  Blocks b{};
  b.n = nb;
  for (int i = 0; i < nb; ++i) {
    b.v[i] = static_cast<const __nv_bfloat16*>(blocks[i]);
    b.dv[i] = static_cast<__nv_bfloat16*>(dblocks[i]);
  }
  check_cuda(cudaFuncSetAttribute(bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm),
             "attn_res smem");
  bwd_kernel<<<grid_for(T), NT, sm, s>>>(b, u, static_cast<const __nv_bfloat16*>(dout), du, T, D, eps);
  check_cuda(cudaGetLastError(), "attn_res bwd launch");
}

}  // namespace ttb
