// Memory-bound sm_100a kernels: RMSNorm fwd/bwd, rotary embedding, SwiGLU.
// All use 16-byte vector accesses (8 bf16 per thread per access); fp32 math.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "launch_api.h"

namespace ttb {
namespace {

using bf16 = __nv_bfloat16;

struct alignas(16) V8 {
  __nv_bfloat162 h[4];
};

__device__ __forceinline__ void load8(const bf16* p, float (&f)[8]) {
  V8 v = *reinterpret_cast<const V8*>(p);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(v.h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ void store8(bf16* p, const float (&f)[8]) {
  V8 v;
#pragma unroll
  for (int i = 0; i < 4; ++i) v.h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  *reinterpret_cast<V8*>(p) = v;
}

__device__ __forceinline__ void loadw8(const void* w, int w_fp32, int64_t idx, float (&f)[8]) {
  if (w_fp32) {
    const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(w) + idx);
    float4 a = p[0], b = p[1];
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  } else {
    load8(static_cast<const bf16*>(w) + idx, f);
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <int NT>
__device__ __forceinline__ float block_sum(float v, float* scratch) {
  v = warp_sum(v);
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  if (l == 0) scratch[w] = v;
  __syncthreads();
  float t = (threadIdx.x < NT / 32) ? scratch[threadIdx.x] : 0.f;
  if (w == 0) t = warp_sum(t);
  if (threadIdx.x == 0) scratch[0] = t;
  __syncthreads();
  float r = scratch[0];
  __syncthreads();
  return r;
}

__device__ __forceinline__ void unpack8(const V8& v, float (&f)[8]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(v.h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

// RMSNorm: a group of WPR warps owns one row at a time (no CTA-wide barrier); each lane keeps
// VPL 16-byte vectors of the row packed in registers, so one row is read once and written once.
// Groups stride over rows (persistent grid); the sum of squares (forward) or of dy*w*x
// (backward) is reduced by shuffles and, for WPR > 1, through a double-buffered shared slot
// with one named barrier per row and group. The backward keeps the weight-gradient partial sums
// of its columns in registers and writes one partial row per group at the end.
constexpr int kNormThreads = 256;

template <int WPR>
__device__ __forceinline__ float group_sum(float v, float (*slot)[8], int parity, int group, int sub) {
  v = warp_sum(v);
  if constexpr (WPR == 1) {
    return v;
  } else {
    if ((threadIdx.x & 31) == 0) slot[parity][group * WPR + sub] = v;
    asm volatile("bar.sync %0, %1;" ::"r"(1 + group), "r"(32 * WPR) : "memory");
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < WPR; ++k) t += slot[parity][group * WPR + k];
    return t;
  }
}

template <int WPR, int VPL, bool BWD, int MINB>
__global__ void __launch_bounds__(kNormThreads, MINB) rmsnorm_rows_kernel(
    const bf16* __restrict__ x, const bf16* __restrict__ dy, const void* __restrict__ w, float* __restrict__ rstd,
    bf16* __restrict__ out, float* __restrict__ dw_partial, int64_t rows, int dim, float eps, int w_fp32) {
  constexpr int kGroups = kNormThreads / 32 / WPR;
  __shared__ float slot[2][8];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int group = warp / WPR, sub = warp % WPR;
  const int v0 = sub * 32 + lane;  // this lane's first vector; the others follow every 32*WPR
  float dwacc[BWD ? VPL : 1][8];
  if constexpr (BWD) {
#pragma unroll
    for (int i = 0; i < VPL; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) dwacc[i][j] = 0.f;
  }
  int parity = 0;
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * kGroups + group; row < rows;
       row += static_cast<int64_t>(gridDim.x) * kGroups, parity ^= 1) {
    V8 xv8[VPL], gv8[BWD ? VPL : 1];
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int c = (v0 + i * 32 * WPR) * 8;
      if (c < dim) {
        xv8[i] = *reinterpret_cast<const V8*>(x + row * dim + c);
        if constexpr (BWD) gv8[i] = *reinterpret_cast<const V8*>(dy + row * dim + c);
      }
    }
    const float r_in = BWD ? rstd[row] : 0.f;
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int c = (v0 + i * 32 * WPR) * 8;
      if (c < dim) {
        float xv[8];
        unpack8(xv8[i], xv);
        if constexpr (BWD) {
          float gv[8], wf[8];
          unpack8(gv8[i], gv);
          loadw8(w, w_fp32, c, wf);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float xh = xv[j] * r_in;
            acc += gv[j] * wf[j] * xh;
            dwacc[i][j] += gv[j] * xh;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) acc += xv[j] * xv[j];
        }
      }
    }
    acc = group_sum<WPR>(acc, slot, parity, group, sub);
    const float r = BWD ? r_in : rsqrtf(acc / dim + eps);
    const float dot = BWD ? acc / dim : 0.f;
    if (!BWD && sub == 0 && lane == 0) rstd[row] = r;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int c = (v0 + i * 32 * WPR) * 8;
      if (c < dim) {
        float xv[8], wf[8], o[8];
        unpack8(xv8[i], xv);
        loadw8(w, w_fp32, c, wf);
        if constexpr (BWD) {
          float gv[8];
          unpack8(gv8[i], gv);
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] = r * (gv[j] * wf[j] - xv[j] * r * dot);
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] = xv[j] * r * wf[j];
        }
        store8(out + row * dim + c, o);
      }
    }
  }
  if constexpr (BWD) {
    float* dst_row = dw_partial + (static_cast<int64_t>(blockIdx.x) * kGroups + group) * dim;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int c = (v0 + i * 32 * WPR) * 8;
      if (c < dim) {
        float4* dst = reinterpret_cast<float4*>(dst_row + c);
        dst[0] = make_float4(dwacc[i][0], dwacc[i][1], dwacc[i][2], dwacc[i][3]);
        dst[1] = make_float4(dwacc[i][4], dwacc[i][5], dwacc[i][6], dwacc[i][7]);
      }
    }
  }
}

// Column sums of a [nparts, dim] fp32 matrix: 32 columns per CTA, 8 warps split the rows and
// combine through shared memory (coalesced 128-byte row segments per warp).
__global__ void __launch_bounds__(256) reduce_rows_kernel(const float* __restrict__ p, float* __restrict__ out,
                                                         int64_t nparts, int64_t dim) {
  __shared__ float part[8][33];
  const int lane = threadIdx.x % 32, wp = threadIdx.x / 32;
  const int64_t c = blockIdx.x * 32LL + lane;
  float s = 0.f;
  if (c < dim)
    for (int64_t i = wp; i < nparts; i += 8) s += p[i * dim + c];
  part[wp][lane] = s;
  __syncthreads();
  if (wp == 0) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) t += part[k][lane];
    if (c < dim) out[c] = t;
  }
}

// x: [B,S,H,D] bf16 contiguous; rotate interleaved pairs (2i, 2i+1) by angle
// table cos/sin[(b,) s, i].  One thread per 8 elements (4 pairs).
__global__ void rope_kernel(const bf16* __restrict__ x, bf16* __restrict__ y, const float* __restrict__ cosT,
                            const float* __restrict__ sinT, int64_t total8, int S, int H, int D, int64_t cs_bstride,
                            float sgn) {
  const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (t >= total8) return;
  const int64_t e = t * 8;
  const int d = static_cast<int>(e % D);
  const int64_t tok = e / ((int64_t)D * H);  // b*S + s
  const int s = static_cast<int>(tok % S);
  const int64_t b = tok / S;
  const float* cp = cosT + b * cs_bstride + (int64_t)s * (D / 2) + d / 2;
  const float* sp = sinT + b * cs_bstride + (int64_t)s * (D / 2) + d / 2;
  float f[8], o[8];
  load8(x + e, f);
  const float4 c4 = *reinterpret_cast<const float4*>(cp);
  const float4 s4 = *reinterpret_cast<const float4*>(sp);
  const float cc[4] = {c4.x, c4.y, c4.z, c4.w};
  const float ss[4] = {s4.x * sgn, s4.y * sgn, s4.z * sgn, s4.w * sgn};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    o[2 * i] = f[2 * i] * cc[i] - f[2 * i + 1] * ss[i];
    o[2 * i + 1] = f[2 * i] * ss[i] + f[2 * i + 1] * cc[i];
  }
  store8(y + e, o);
}

__device__ __forceinline__ float sigmoidf_(float a) { return 1.f / (1.f + __expf(-a)); }

__global__ void swiglu_fwd_kernel(const bf16* __restrict__ a, const bf16* __restrict__ b, bf16* __restrict__ y,
                                  int64_t n8) {
  const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (t >= n8) return;
  float fa[8], fb[8], o[8];
  load8(a + t * 8, fa);
  load8(b + t * 8, fb);
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j] = fa[j] * sigmoidf_(fa[j]) * fb[j];
  store8(y + t * 8, o);
}

__global__ void swiglu_bwd_kernel(const bf16* __restrict__ dy, const bf16* __restrict__ a, const bf16* __restrict__ b,
                                  bf16* __restrict__ da, bf16* __restrict__ db, int64_t n8) {
  const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (t >= n8) return;
  float g[8], fa[8], fb[8], oa[8], ob[8];
  load8(dy + t * 8, g);
  load8(a + t * 8, fa);
  load8(b + t * 8, fb);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float sg = sigmoidf_(fa[j]);
    const float silu = fa[j] * sg;
    ob[j] = g[j] * silu;
    oa[j] = g[j] * fb[j] * sg * (1.f + fa[j] * (1.f - sg));
  }
  store8(da + t * 8, oa);
  store8(db + t * 8, ob);
}

// out[p] = src[idx[p]] (idx < 0: a zero row); bf16 rows of d elements, 16-byte vectors, one
// warp per output row
__global__ void __launch_bounds__(256) gather_rows_kernel(const bf16* __restrict__ src, const int64_t* __restrict__ idx,
                                                          bf16* __restrict__ out, int64_t rows, int d8,
                                                          int64_t n_src) {
  const int64_t p = static_cast<int64_t>(blockIdx.x) * 8 + threadIdx.x / 32;
  if (p >= rows) return;
  const int64_t sr = idx[p];
  const int lane = threadIdx.x % 32;
  V8* o = reinterpret_cast<V8*>(out) + p * d8;
  if (sr < 0 || sr >= n_src) {  // (an index past the source also reads as a zero row)
    V8 z;
    for (int i = 0; i < 4; ++i) z.h[i] = __floats2bfloat162_rn(0.f, 0.f);
    for (int c = lane; c < d8; c += 32) o[c] = z;
  } else {
    const V8* s = reinterpret_cast<const V8*>(src) + sr * d8;
    for (int c = lane; c < d8; c += 32) o[c] = s[c];
  }
}

// Row-group shapes: (warps per row, vectors per lane, resident CTAs per SM). The forward keeps
// up to 8 vectors (128 bytes) of x per lane, the backward up to 4 of x and 4 of dy (plus the
// 32 fp32 weight-gradient sums); 16384-wide rows use 8 warps and 8 vectors.
struct NormShape {
  int wpr, vpl, minb;
};
NormShape norm_shape(int64_t dim, bool bwd) {
  const int64_t vecs = dim / 8;
  const int cap = bwd ? 4 : 8;
  int wpr = 1;
  while (wpr < 8 && vecs > 32LL * wpr * cap) wpr *= 2;
  int vpl = static_cast<int>((vecs + 32LL * wpr - 1) / (32LL * wpr));
  vpl = vpl <= 1 ? 1 : vpl <= 2 ? 2 : vpl <= 4 ? 4 : 8;
  const int minb = bwd ? (vpl <= 2 ? 4 : (vpl == 4 ? 2 : 1)) : (vpl <= 4 ? 4 : 3);
  return {wpr, vpl, minb};
}

template <int WPR, int VPL, bool BWD, int MINB>
void launch_rows(const void* x, const void* dy, const void* w, float* rstd, void* out, float* dwp, int64_t rows,
                 int64_t dim, float eps, int w_fp32, int grid, cudaStream_t s) {
  rmsnorm_rows_kernel<WPR, VPL, BWD, MINB><<<static_cast<unsigned>(grid), kNormThreads, 0, s>>>(
      static_cast<const bf16*>(x), static_cast<const bf16*>(dy), w, rstd, static_cast<bf16*>(out), dwp, rows,
      static_cast<int>(dim), eps, w_fp32);
}

template <bool BWD>
void dispatch_rows(const void* x, const void* dy, const void* w, float* rstd, void* out, float* dwp, int64_t rows,
                   int64_t dim, float eps, int w_fp32, int grid, cudaStream_t s) {
  const NormShape sh = norm_shape(dim, BWD);
#define TTB_NORM_CASE(W, V, M)                                                                \
  if (sh.wpr == W && sh.vpl == V && sh.minb == M) {                                           \
    launch_rows<W, V, BWD, M>(x, dy, w, rstd, out, dwp, rows, dim, eps, w_fp32, grid, s); \
    return;                                                                                   \
  }
  if constexpr (BWD) {
    TTB_NORM_CASE(1, 1, 4) TTB_NORM_CASE(1, 2, 4) TTB_NORM_CASE(1, 4, 2) TTB_NORM_CASE(2, 4, 2)
    TTB_NORM_CASE(4, 4, 2) TTB_NORM_CASE(8, 4, 2) TTB_NORM_CASE(8, 8, 1)
  } else {
    TTB_NORM_CASE(1, 1, 4) TTB_NORM_CASE(1, 2, 4) TTB_NORM_CASE(1, 4, 4) TTB_NORM_CASE(1, 8, 3)
    TTB_NORM_CASE(2, 8, 3) TTB_NORM_CASE(4, 8, 3) TTB_NORM_CASE(8, 8, 3)
  }
#undef TTB_NORM_CASE
  throw std::runtime_error("rmsnorm: no kernel for this width");
}

int norm_grid(int64_t rows, int64_t dim, bool bwd, int sms) {
  const NormShape sh = norm_shape(dim, bwd);
  const int64_t groups = kNormThreads / 32 / sh.wpr;
  const int64_t need = (rows + groups - 1) / groups;
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(need, static_cast<int64_t>(sms) * sh.minb)));
}

}  // namespace

void rmsnorm_fwd(const void* x, const void* w, void* y, float* rstd, int64_t rows, int64_t dim, float eps, int w_fp32,
                 cudaStream_t s) {
  if (dim % 8) throw std::runtime_error("rmsnorm: dim must be a multiple of 8");
  if (dim > 16384) throw std::runtime_error("rmsnorm: dim > 16384 unsupported");
  if (rows == 0) return;
  int dev = 0;
  cudaGetDevice(&dev);
  dispatch_rows<false>(x, nullptr, w, rstd, y, nullptr, rows, dim, eps, w_fp32, norm_grid(rows, dim, false, num_sms(dev)),
                       s);
  check_cuda(cudaGetLastError(), "rmsnorm_fwd");
}

int rmsnorm_bwd_parts(int64_t rows, int64_t dim, int sms) {
  return norm_grid(rows, dim, true, sms) * (kNormThreads / 32 / norm_shape(dim, true).wpr);
}

void rmsnorm_bwd(const void* dy, const void* x, const void* w, const float* rstd, void* dx, float* dw_partial,
                 int64_t rows, int64_t dim, int w_fp32, int nparts, cudaStream_t s) {
  if (dim % 8) throw std::runtime_error("rmsnorm: dim must be a multiple of 8");
  if (dim > 16384) throw std::runtime_error("rmsnorm: dim > 16384 unsupported");
  const int groups = kNormThreads / 32 / norm_shape(dim, true).wpr;
  if (nparts % groups) throw std::runtime_error("rmsnorm_bwd: partial rows must come from rmsnorm_bwd_parts");
  dispatch_rows<true>(x, dy, w, const_cast<float*>(rstd), dx, dw_partial, rows, dim, 0.f, w_fp32, nparts / groups,
                      s);
  check_cuda(cudaGetLastError(), "rmsnorm_bwd");
}

void gather_rows_bf16(const void* src, int64_t n_src, const int64_t* idx, void* out, int64_t rows, int64_t d,
                      cudaStream_t s) {
  if (d % 8) throw std::runtime_error("gather_rows: row length must be a multiple of 8");
  if (rows == 0) return;
  gather_rows_kernel<<<static_cast<unsigned>((rows + 7) / 8), 256, 0, s>>>(
      static_cast<const bf16*>(src), idx, static_cast<bf16*>(out), rows, static_cast<int>(d / 8), n_src);
  check_cuda(cudaGetLastError(), "gather_rows");
}

void reduce_rows_f32(const float* partial, float* out, int64_t nparts, int64_t dim, cudaStream_t s) {
  reduce_rows_kernel<<<static_cast<unsigned>((dim + 31) / 32), 256, 0, s>>>(partial, out, nparts, dim);
  check_cuda(cudaGetLastError(), "reduce_rows");
}

void rope_apply(const void* x, void* y, const float* cos, const float* sin, int64_t B, int64_t S, int64_t H,
                int64_t D, int64_t cs_batch_stride, bool inverse, cudaStream_t s) {
  if (D % 8) throw std::runtime_error("rope: head_dim must be a multiple of 8");
  const int64_t total8 = B * S * H * D / 8;
  if (total8 == 0) return;
  rope_kernel<<<static_cast<unsigned>((total8 + 255) / 256), 256, 0, s>>>(
      static_cast<const bf16*>(x), static_cast<bf16*>(y), cos, sin, total8, (int)S, (int)H, (int)D, cs_batch_stride,
      inverse ? -1.f : 1.f);
  check_cuda(cudaGetLastError(), "rope");
}

void swiglu_fwd(const void* a, const void* b, void* y, int64_t n, cudaStream_t s) {
  if (n % 8) throw std::runtime_error("swiglu: numel must be a multiple of 8");
  const int64_t n8 = n / 8;
  if (n8 == 0) return;
  swiglu_fwd_kernel<<<static_cast<unsigned>((n8 + 255) / 256), 256, 0, s>>>(
      static_cast<const bf16*>(a), static_cast<const bf16*>(b), static_cast<bf16*>(y), n8);
  check_cuda(cudaGetLastError(), "swiglu_fwd");
}

void swiglu_bwd(const void* dy, const void* a, const void* b, void* da, void* db, int64_t n, cudaStream_t s) {
  if (n % 8) throw std::runtime_error("swiglu: numel must be a multiple of 8");
  const int64_t n8 = n / 8;
  if (n8 == 0) return;
  swiglu_bwd_kernel<<<static_cast<unsigned>((n8 + 255) / 256), 256, 0, s>>>(
      static_cast<const bf16*>(dy), static_cast<const bf16*>(a), static_cast<const bf16*>(b), static_cast<bf16*>(da),
      static_cast<bf16*>(db), n8);
  check_cuda(cudaGetLastError(), "swiglu_bwd");
}

}  // namespace ttb
