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

// One CTA per row; each thread owns VPT vectors of 8 elements kept in registers.
template <int NT, int VPT>
__global__ void __launch_bounds__(NT) rmsnorm_fwd_kernel(const bf16* __restrict__ x, const void* __restrict__ w,
                                                         bf16* __restrict__ y, float* __restrict__ rstd_out, int dim,
                                                         float eps, int w_fp32) {
  __shared__ float scratch[32];
  const int64_t row = blockIdx.x;
  const bf16* xr = x + row * dim;
  float v[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (threadIdx.x + i * NT) * 8;
    if (c < dim) {
      load8(xr + c, v[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
    }
  }
  ss = block_sum<NT>(ss, scratch);
  const float r = rsqrtf(ss / dim + eps);
  if (threadIdx.x == 0) rstd_out[row] = r;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (threadIdx.x + i * NT) * 8;
    if (c < dim) {
      float wf[8], o[8];
      loadw8(w, w_fp32, c, wf);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = v[i][j] * r * wf[j];
      store8(y + row * dim + c, o);
    }
  }
}

// Persistent CTAs stride over rows; dw partial sums per CTA in registers.
template <int NT, int VPT>
__global__ void __launch_bounds__(NT) rmsnorm_bwd_kernel(const bf16* __restrict__ dy, const bf16* __restrict__ x,
                                                         const void* __restrict__ w, const float* __restrict__ rstd,
                                                         bf16* __restrict__ dx, float* __restrict__ dw_partial,
                                                         int64_t rows, int dim, int w_fp32) {
  __shared__ float scratch[32];
  float dwacc[VPT][8];
  float wf[VPT][8];
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (threadIdx.x + i * NT) * 8;
#pragma unroll
    for (int j = 0; j < 8; ++j) dwacc[i][j] = 0.f;
    if (c < dim) loadw8(w, w_fp32, c, wf[i]);
  }
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const float r = rstd[row];
    float xv[VPT][8], gv[VPT][8];
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = (threadIdx.x + i * NT) * 8;
      if (c < dim) {
        load8(x + row * dim + c, xv[i]);
        load8(dy + row * dim + c, gv[i]);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float xh = xv[i][j] * r;
          dot += gv[i][j] * wf[i][j] * xh;
          dwacc[i][j] += gv[i][j] * xh;
        }
      }
    }
    dot = block_sum<NT>(dot, scratch) / dim;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = (threadIdx.x + i * NT) * 8;
      if (c < dim) {
        float o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = r * (gv[i][j] * wf[i][j] - xv[i][j] * r * dot);
        store8(dx + row * dim + c, o);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (threadIdx.x + i * NT) * 8;
    if (c < dim) {
      float* dst = dw_partial + static_cast<int64_t>(blockIdx.x) * dim + c;
#pragma unroll
      for (int j = 0; j < 8; ++j) dst[j] = dwacc[i][j];
    }
  }
}

__global__ void reduce_rows_kernel(const float* __restrict__ p, float* __restrict__ out, int64_t nparts, int64_t dim) {
  const int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (c >= dim) return;
  float s = 0.f;
  for (int64_t i = 0; i < nparts; ++i) s += p[i * dim + c];
  out[c] = s;
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

template <int NT, int VPT>
void launch_fwd(const void* x, const void* w, void* y, float* rstd, int64_t rows, int64_t dim, float eps, int w_fp32,
                cudaStream_t s) {
  rmsnorm_fwd_kernel<NT, VPT><<<static_cast<unsigned>(rows), NT, 0, s>>>(
      static_cast<const bf16*>(x), w, static_cast<bf16*>(y), rstd, static_cast<int>(dim), eps, w_fp32);
}

template <int NT, int VPT>
void launch_bwd(const void* dy, const void* x, const void* w, const float* rstd, void* dx, float* dwp, int64_t rows,
                int64_t dim, int w_fp32, int nparts, cudaStream_t s) {
  rmsnorm_bwd_kernel<NT, VPT><<<nparts, NT, 0, s>>>(static_cast<const bf16*>(dy), static_cast<const bf16*>(x), w,
                                                    rstd, static_cast<bf16*>(dx), dwp, rows, static_cast<int>(dim),
                                                    w_fp32);
}

}  // namespace

void rmsnorm_fwd(const void* x, const void* w, void* y, float* rstd, int64_t rows, int64_t dim, float eps, int w_fp32,
                 cudaStream_t s) {
  if (dim % 8) throw std::runtime_error("rmsnorm: dim must be a multiple of 8");
  const int64_t vecs = dim / 8;
  if (rows == 0) return;
  if (vecs <= 128) launch_fwd<128, 1>(x, w, y, rstd, rows, dim, eps, w_fp32, s);
  else if (vecs <= 256) launch_fwd<256, 1>(x, w, y, rstd, rows, dim, eps, w_fp32, s);
  else if (vecs <= 512) launch_fwd<256, 2>(x, w, y, rstd, rows, dim, eps, w_fp32, s);
  else if (vecs <= 1024) launch_fwd<256, 4>(x, w, y, rstd, rows, dim, eps, w_fp32, s);
  else if (vecs <= 2048) launch_fwd<512, 4>(x, w, y, rstd, rows, dim, eps, w_fp32, s);
  else throw std::runtime_error("rmsnorm: dim > 16384 unsupported");
  check_cuda(cudaGetLastError(), "rmsnorm_fwd");
}

void rmsnorm_bwd(const void* dy, const void* x, const void* w, const float* rstd, void* dx, float* dw_partial,
                 int64_t rows, int64_t dim, int w_fp32, int nparts, cudaStream_t s) {
  if (dim % 8) throw std::runtime_error("rmsnorm: dim must be a multiple of 8");
  const int64_t vecs = dim / 8;
  if (vecs <= 128) launch_bwd<128, 1>(dy, x, w, rstd, dx, dw_partial, rows, dim, w_fp32, nparts, s);
  else if (vecs <= 256) launch_bwd<256, 1>(dy, x, w, rstd, dx, dw_partial, rows, dim, w_fp32, nparts, s);
  else if (vecs <= 512) launch_bwd<256, 2>(dy, x, w, rstd, dx, dw_partial, rows, dim, w_fp32, nparts, s);
  else if (vecs <= 1024) launch_bwd<256, 4>(dy, x, w, rstd, dx, dw_partial, rows, dim, w_fp32, nparts, s);
  else if (vecs <= 2048) launch_bwd<512, 4>(dy, x, w, rstd, dx, dw_partial, rows, dim, w_fp32, nparts, s);
  else throw std::runtime_error("rmsnorm: dim > 16384 unsupported");
  check_cuda(cudaGetLastError(), "rmsnorm_bwd");
}

void reduce_rows_f32(const float* partial, float* out, int64_t nparts, int64_t dim, cudaStream_t s) {
  reduce_rows_kernel<<<static_cast<unsigned>((dim + 255) / 256), 256, 0, s>>>(partial, out, nparts, dim);
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
