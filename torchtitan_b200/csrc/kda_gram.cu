// Decayed Gram matrices of the chunked KDA (Kimi Delta Attention) forward and
// backward, one CTA per (sequence, head, chunk):
//
//   out[i,j] = sum_d a[i,d] b[j,d] exp(min(G[i,d] - G[j,d], 0))   for j < i (strict) or j <= i
//
// G is the within-chunk cumulative log decay (non-increasing in i), so every
// exponent is <= 0: the pairwise form never overflows (unlike exp(G_i) *
// exp(-G_j)).  Backward, with w = dout masked to the same triangle and
// e = exp(min(G_i - G_j, 0)):
//   da[i,d] = sum_j w[i,j] e b[j,d]
//   db[j,d] = sum_i w[i,j] e a[i,d]
//   dG[i,d] = a[i,d] da[i,d] - b[i,d] db[i,d]
// (the last line collects d/dG of e through both of its indices).  Tiles live in
// shared memory with one padding word per row (bank-conflict free column walks).
#include <cuda_runtime.h>

#include <stdexcept>

#include "launch_api.h"

namespace ttb {
namespace kda_impl {

constexpr int NT = 256;

__device__ __forceinline__ float decay(float gi, float gj) { return __expf(fminf(gi - gj, 0.f)); }

__global__ void __launch_bounds__(NT) gram_fwd_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                                      const float* __restrict__ G, float* __restrict__ out, int C,
                                                      int K, int strict) {
  extern __shared__ float sm[];
  const int P = K + 1;
  float* sa = sm;
  float* sb = sa + C * P;
  float* sg = sb + C * P;
  const size_t base = static_cast<size_t>(blockIdx.x) * C * K;
  for (int x = threadIdx.x; x < C * K; x += NT) {
    const int r = x / K, d = x - r * K;
    sa[r * P + d] = a[base + x];
    sb[r * P + d] = b[base + x];
    sg[r * P + d] = G[base + x];
  }
  __syncthreads();
  float* o = out + static_cast<size_t>(blockIdx.x) * C * C;
  for (int x = threadIdx.x; x < C * C; x += NT) {
    const int i = x / C, j = x - i * C;
    float acc = 0.f;
    if (strict ? j < i : j <= i) {
      const float* ai = sa + i * P;
      const float* gi = sg + i * P;
      const float* bj = sb + j * P;
      const float* gj = sg + j * P;
#pragma unroll 4
      for (int d = 0; d < K; ++d) acc += ai[d] * bj[d] * decay(gi[d], gj[d]);
    }
    o[x] = acc;
  }
}

__global__ void __launch_bounds__(NT) gram_bwd_kernel(const float* __restrict__ dout, const float* __restrict__ a,
                                                      const float* __restrict__ b, const float* __restrict__ G,
                                                      float* __restrict__ da, float* __restrict__ db,
                                                      float* __restrict__ dG, int C, int K, int strict) {
  extern __shared__ float sm[];
  const int P = K + 1;
  float* sa = sm;
  float* sb = sa + C * P;
  float* sg = sb + C * P;
  float* sw = sg + C * P;  // [C, C + 1] masked upstream gradient
  const size_t base = static_cast<size_t>(blockIdx.x) * C * K;
  for (int x = threadIdx.x; x < C * K; x += NT) {
    const int r = x / K, d = x - r * K;
    sa[r * P + d] = a[base + x];
    sb[r * P + d] = b[base + x];
    sg[r * P + d] = G[base + x];
  }
  const float* w = dout + static_cast<size_t>(blockIdx.x) * C * C;
  for (int x = threadIdx.x; x < C * C; x += NT) {
    const int i = x / C, j = x - i * C;
    sw[i * (C + 1) + j] = (strict ? j < i : j <= i) ? w[x] : 0.f;
  }
  __syncthreads();
  // threads walk d fastest: consecutive threads read consecutive words of a row
  for (int x = threadIdx.x; x < C * K; x += NT) {
    const int r = x / K, d = x - r * K;
    const float gr = sg[r * P + d];
    float s_row = 0.f, s_col = 0.f;  // da[r,d] (r as i), db[r,d] (r as j)
    for (int t = 0; t < C; ++t) {
      const float gt = sg[t * P + d];
      s_row += sw[r * (C + 1) + t] * decay(gr, gt) * sb[t * P + d];
      s_col += sw[t * (C + 1) + r] * decay(gt, gr) * sa[t * P + d];
    }
    da[base + x] = s_row;
    db[base + x] = s_col;
    dG[base + x] = sa[r * P + d] * s_row - sb[r * P + d] * s_col;
  }
}

size_t smem_bytes(int C, int K, bool bwd) {
  return (static_cast<size_t>(3) * C * (K + 1) + (bwd ? static_cast<size_t>(C) * (C + 1) : 0)) * sizeof(float);
}

}  // namespace kda_impl

void kda_gram_fwd(const float* a, const float* b, const float* G, float* out, int64_t N, int C, int K, bool strict,
                  cudaStream_t s) {
  using namespace kda_impl;
  if (N == 0) return;
  const size_t sm = smem_bytes(C, K, false);
  if (sm > 227 * 1024) throw std::runtime_error("kda_gram: chunk x head dim too large for shared memory");
  check_cuda(cudaFuncSetAttribute(gram_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm),
             "kda gram smem");
  gram_fwd_kernel<<<(unsigned)N, NT, sm, s>>>(a, b, G, out, C, K, strict ? 1 : 0);
  check_cuda(cudaGetLastError(), "kda gram fwd launch");
}

void kda_gram_bwd(const float* dout, const float* a, const float* b, const float* G, float* da, float* db,
                  float* dG, int64_t N, int C, int K, bool strict, cudaStream_t s) {
  using namespace kda_impl;
  if (N == 0) return;
  const size_t sm = smem_bytes(C, K, true);
  if (sm > 227 * 1024) throw std::runtime_error("kda_gram: chunk x head dim too large for shared memory");
  check_cuda(cudaFuncSetAttribute(gram_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm),
             "kda gram smem");
  gram_bwd_kernel<<<(unsigned)N, NT, sm, s>>>(dout, a, b, G, da, db, dG, C, K, strict ? 1 : 0);
  check_cuda(cudaGetLastError(), "kda gram bwd launch");
}

}  // namespace ttb
