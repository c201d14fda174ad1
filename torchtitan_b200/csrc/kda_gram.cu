// Decayed Gram matrices of the chunked KDA (Kimi Delta Attention) forward and
// backward, one CTA per (sequence, head, chunk):
//
//   out[i,j] = sum_d a[i,d] b[j,d] exp(min(G[i,d] - G[j,d], 0))   for j < i (strict) or j <= i
//
// G is the within-chunk cumulative log decay (non-increasing in i), so every
// exponent is <= 0: the pairwise form never overflows (unlike exp(G_i) *
// exp(-G_j)); the kernels factor it per 16-row sub-chunk so that both factors
// stay <= 1.  Backward, with w = dout masked to the same triangle and
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

constexpr int NT = 512;
constexpr int SUB = 16;  // sub-chunk rows sharing one reference point of the factorised decay

__device__ __forceinline__ float decay(float gi, float gj) { return __expf(fminf(gi - gj, 0.f)); }

// Factorised decay between sub-chunks. With r = G[16I] (first row of sub-chunk I) and G
// non-increasing along the chunk, for i in I and j < 16I:
//   exp(G_i - G_j) = exp(G_i - r) * exp(r - G_j),   both factors in (0, 1]
// so the off-diagonal blocks are plain dot products of pre-scaled rows (one exponential per
// row element instead of one per (i, j, d) triple) and nothing can overflow. The diagonal
// 16x16 blocks keep the exact pairwise form (with its clamp at 0).
//
// Shared layout (row pitch P = K + 1 words): a, b, G [C rows] | scaled-a [SUB rows] |
// scaled-b [C - SUB rows] (| masked dout [C x (C + 1)] in the backward).
__device__ __forceinline__ void load_tiles(const float* a, const float* b, const float* G, float* sa, float* sb,
                                           float* sg, size_t base, int C, int K, int P) {
  // 16-byte loads, eight per tensor issued before any is stored (the tiles are 16-byte
  // aligned: base is a multiple of C * K and K % 4 == 0)
  const int n4 = C * K / 4;
  for (int x0 = threadIdx.x; x0 < n4; x0 += 8 * NT) {
    float4 va[8], vb[8], vg[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int x = x0 + u * NT;
      if (x < n4) {
        va[u] = reinterpret_cast<const float4*>(a + base)[x];
        vb[u] = reinterpret_cast<const float4*>(b + base)[x];
        vg[u] = reinterpret_cast<const float4*>(G + base)[x];
      }
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int x = x0 + u * NT;
      if (x < n4) {
        const int e = 4 * x, r = e / K, d = e - r * K;
        float* pa = sa + r * P + d;
        float* pb = sb + r * P + d;
        float* pg = sg + r * P + d;
        pa[0] = va[u].x; pa[1] = va[u].y; pa[2] = va[u].z; pa[3] = va[u].w;
        pb[0] = vb[u].x; pb[1] = vb[u].y; pb[2] = vb[u].z; pb[3] = vb[u].w;
        pg[0] = vg[u].x; pg[1] = vg[u].y; pg[2] = vg[u].z; pg[3] = vg[u].w;
      }
    }
  }
}

// scaled rows for sub-chunk I: ta[i'] = a[16I + i'] exp(G - r), tb[j] = b[j] exp(r - G), j < 16I
__device__ __forceinline__ void scale_rows(const float* sa, const float* sb, const float* sg, float* ta, float* tb,
                                           int I, int K, int P) {
  const int r0 = I * SUB;
  for (int x = threadIdx.x; x < (SUB + r0) * K; x += NT) {
    const int row = x / K, d = x - row * K;
    const float ref = sg[r0 * P + d];
    if (row < SUB) {
      const int i = r0 + row;
      ta[row * P + d] = sa[i * P + d] * __expf(fminf(sg[i * P + d] - ref, 0.f));
    } else {
      const int j = row - SUB;
      tb[j * P + d] = sb[j * P + d] * __expf(fminf(ref - sg[j * P + d], 0.f));
    }
  }
}

__global__ void __launch_bounds__(NT) gram_fwd_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                                      const float* __restrict__ G, float* __restrict__ out, int C,
                                                      int K, int strict) {
  extern __shared__ float sm[];
  const int P = K + 1;
  float* sa = sm;
  float* sb = sa + C * P;
  float* sg = sb + C * P;
  float* ta = sg + C * P;
  float* tb = ta + SUB * P;
  const size_t base = static_cast<size_t>(blockIdx.x) * C * K;
  load_tiles(a, b, G, sa, sb, sg, base, C, K, P);
  float* o = out + static_cast<size_t>(blockIdx.x) * C * C;
  // everything right of the diagonal block is zero
  for (int x = threadIdx.x; x < C * C; x += NT) {
    const int i = x / C, j = x - i * C;
    if (j / SUB > i / SUB) o[x] = 0.f;
  }
  for (int I = 0; I < C / SUB; ++I) {
    __syncthreads();  // tiles loaded / previous sub-chunk's scaled rows consumed
    scale_rows(sa, sb, sg, ta, tb, I, K, P);
    __syncthreads();
    const int r0 = I * SUB;
    // columns j < 16I: factorised dot products, 2x2 outputs per thread (four independent
    // accumulators, one shared-memory load per FMA)
    for (int x = threadIdx.x; x < (SUB / 2) * (r0 / 2); x += NT) {
      const int ip = x / (r0 / 2), jp = x - ip * (r0 / 2);
      const float* a0 = ta + (2 * ip) * P;
      const float* a1 = a0 + P;
      const float* b0 = tb + (2 * jp) * P;
      const float* b1 = b0 + P;
      float c00 = 0.f, c01 = 0.f, c10 = 0.f, c11 = 0.f;
#pragma unroll 4
      for (int d = 0; d < K; ++d) {
        const float x0 = a0[d], x1 = a1[d], y0 = b0[d], y1 = b1[d];
        c00 = fmaf(x0, y0, c00);
        c01 = fmaf(x0, y1, c01);
        c10 = fmaf(x1, y0, c10);
        c11 = fmaf(x1, y1, c11);
      }
      const int i = r0 + 2 * ip, j = 2 * jp;
      o[i * C + j] = c00;
      o[i * C + j + 1] = c01;
      o[(i + 1) * C + j] = c10;
      o[(i + 1) * C + j + 1] = c11;
    }
    // the diagonal block: exact pairwise decay, four partial sums over d
    for (int x = threadIdx.x; x < SUB * SUB; x += NT) {
      const int i = r0 + x / SUB, j = r0 + x % SUB;
      float p0 = 0.f, p1 = 0.f, p2 = 0.f, p3 = 0.f;
      if (strict ? j < i : j <= i) {
        const float* ai = sa + i * P;
        const float* gi = sg + i * P;
        const float* bj = sb + j * P;
        const float* gj = sg + j * P;
        for (int d = 0; d < K; d += 4) {
          p0 += ai[d] * bj[d] * decay(gi[d], gj[d]);
          p1 += ai[d + 1] * bj[d + 1] * decay(gi[d + 1], gj[d + 1]);
          p2 += ai[d + 2] * bj[d + 2] * decay(gi[d + 2], gj[d + 2]);
          p3 += ai[d + 3] * bj[d + 3] * decay(gi[d + 3], gj[d + 3]);
        }
      }
      o[i * C + j] = (p0 + p1) + (p2 + p3);
    }
  }
}

// Backward with w = dout masked to the triangle, e_ijd = exp(min(G_i - G_j, 0)):
//   da[i,d] = sum_j w[i,j] e b[j,d],  db[j,d] = sum_i w[i,j] e a[i,d],  dG = a da - b db
// Off-diagonal blocks by the same factorisation: for i in I, j < 16I,
//   da[i,d] += exp(G_i - r) sum_j w[i,j] tb[j,d],   db[j,d] += exp(r - G_j) sum_i w[i,j] ta'[i,d]
// where ta' = a[i] exp(G_i - r) (the forward's scaled a).
__global__ void __launch_bounds__(NT) gram_bwd_kernel(const float* __restrict__ dout, const float* __restrict__ a,
                                                      const float* __restrict__ b, const float* __restrict__ G,
                                                      float* __restrict__ da, float* __restrict__ db,
                                                      float* __restrict__ dG, int C, int K, int strict) {
  extern __shared__ float sm[];
  const int P = K + 1;
  float* sa = sm;
  float* sb = sa + C * P;
  float* sg = sb + C * P;
  float* ta = sg + C * P;
  float* tb = ta + SUB * P;
  float* sw = tb + (C - SUB) * P;  // [C, C + 1] masked upstream gradient
  float* sda = sw + C * (C + 1);   // [C, P] accumulators
  float* sdb = sda + C * P;
  const size_t base = static_cast<size_t>(blockIdx.x) * C * K;
  load_tiles(a, b, G, sa, sb, sg, base, C, K, P);
  const float* w = dout + static_cast<size_t>(blockIdx.x) * C * C;
  for (int x = threadIdx.x; x < C * C; x += NT) {
    const int i = x / C, j = x - i * C;
    sw[i * (C + 1) + j] = (strict ? j < i : j <= i) ? w[x] : 0.f;
  }
  for (int x = threadIdx.x; x < C * K; x += NT) {
    const int r = x / K, d = x - r * K;
    sda[r * P + d] = 0.f;
    sdb[r * P + d] = 0.f;
  }
  for (int I = 0; I < C / SUB; ++I) {
    __syncthreads();
    scale_rows(sa, sb, sg, ta, tb, I, K, P);
    __syncthreads();
    const int r0 = I * SUB;
    // threads walk d fastest over (row, d) elements of rows [0, 16I + 16)
    for (int x = threadIdx.x; x < (r0 + SUB) * K; x += NT) {
      const int r = x / K, d = x - r * K;
      const float gr = sg[r * P + d];
      const float ref = sg[r0 * P + d];
      if (r >= r0) {  // row of sub-chunk I: da from columns j < 16I, diagonal block for da and db
        const float* wr = sw + r * (C + 1);
        float s0 = 0.f, s1 = 0.f;
        for (int j = 0; j < r0; j += 2) {
          s0 = fmaf(wr[j], tb[j * P + d], s0);
          s1 = fmaf(wr[j + 1], tb[(j + 1) * P + d], s1);
        }
        float acc_a = (s0 + s1) * __expf(fminf(gr - ref, 0.f));
        float acc_b = 0.f;
        // one exponential per pair: w[r, t] needs t <= r and w[t, r] needs t >= r, and on
        // those sides the clamped decay is exp(-|G_r - G_t|)
        for (int t = r0; t < r0 + SUB; ++t) {
          const float e = __expf(-fabsf(gr - sg[t * P + d]));
          acc_a = fmaf(wr[t] * e, sb[t * P + d], acc_a);
          acc_b = fmaf(sw[t * (C + 1) + r] * e, sa[t * P + d], acc_b);
        }
        sda[r * P + d] += acc_a;
        sdb[r * P + d] += acc_b;
      } else {  // earlier row j: db from the rows of sub-chunk I
        float s0 = 0.f, s1 = 0.f;
        for (int ii = 0; ii < SUB; ii += 2) {
          s0 = fmaf(sw[(r0 + ii) * (C + 1) + r], ta[ii * P + d], s0);
          s1 = fmaf(sw[(r0 + ii + 1) * (C + 1) + r], ta[(ii + 1) * P + d], s1);
        }
        sdb[r * P + d] += (s0 + s1) * __expf(fminf(ref - gr, 0.f));
      }
    }
  }
  __syncthreads();
  for (int x = threadIdx.x; x < C * K; x += NT) {
    const int r = x / K, d = x - r * K;
    const float va = sda[r * P + d], vb = sdb[r * P + d];
    da[base + x] = va;
    db[base + x] = vb;
    dG[base + x] = sa[r * P + d] * va - sb[r * P + d] * vb;
  }
}

size_t smem_bytes(int C, int K, bool bwd) {
  const size_t P = K + 1;
  size_t words = 3 * C * P + static_cast<size_t>(C) * P;  // a, b, G + scaled a (16 rows) and b (C - 16)
  if (bwd) words += static_cast<size_t>(C) * (C + 1) + 2 * C * P;
  return words * sizeof(float);
}

}  // namespace kda_impl

void kda_gram_fwd(const float* a, const float* b, const float* G, float* out, int64_t N, int C, int K, bool strict,
                  cudaStream_t s) {
  using namespace kda_impl;
  if (N == 0) return;
  if (C % SUB || K % 4) throw std::runtime_error("kda_gram: chunk size must be a multiple of 16, K of 4");
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
  if (C % SUB || K % 4) throw std::runtime_error("kda_gram: chunk size must be a multiple of 16, K of 4");
  const size_t sm = smem_bytes(C, K, true);
  if (sm > 227 * 1024) throw std::runtime_error("kda_gram: chunk x head dim too large for shared memory");
  check_cuda(cudaFuncSetAttribute(gram_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm),
             "kda gram smem");
  gram_bwd_kernel<<<(unsigned)N, NT, sm, s>>>(dout, a, b, G, da, db, dG, C, K, strict ? 1 : 0);
  check_cuda(cudaGetLastError(), "kda gram bwd launch");
}

}  // namespace ttb
