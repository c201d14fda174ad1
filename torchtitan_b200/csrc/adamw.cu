// Multi-tensor AdamW (decoupled weight decay) for sm_100a.
//
// The host flattens every (param, grad, exp_avg, exp_avg_sq) quadruple into
// fixed-size chunks; one launch processes all chunks of all tensors.  Params
// are fp32 (master) or bf16, grads fp32 or bf16, moments fp32.  The chunk
// table travels as a kernel argument in batches, so nothing is allocated on
// the device.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <vector>

#include "launch_api.h"

namespace ttb {
namespace {

constexpr int CHUNK = 65536;
constexpr int MAX_CHUNKS = 320;  // per launch: fits the 32 KB kernel-parameter budget
constexpr int NT = 512;

struct Chunk {
  void* p;
  const void* g;
  float* m;
  float* v;
  int n;
  int8_t p_bf16;
  int8_t g_bf16;
};

struct Table {
  Chunk c[MAX_CHUNKS];
};

__device__ __forceinline__ float ldv(const void* base, int64_t i, int8_t is_bf16) {
  return is_bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(base)[i]) : static_cast<const float*>(base)[i];
}

__global__ void __launch_bounds__(NT) adamw_kernel(const __grid_constant__ Table t, float lr, float b1, float b2,
                                                   float eps, float wd, float bc1, float bc2_sqrt) {
  const Chunk c = t.c[blockIdx.x];
  const float step_size = lr / bc1;
  const float decay = 1.f - lr * wd;
  for (int i = threadIdx.x; i < c.n; i += NT) {
    const float g = ldv(c.g, i, c.g_bf16);
    float m = c.m[i], v = c.v[i];
    m = b1 * m + (1.f - b1) * g;
    v = b2 * v + (1.f - b2) * g * g;
    c.m[i] = m;
    c.v[i] = v;
    const float denom = sqrtf(v) / bc2_sqrt + eps;
    if (c.p_bf16) {
      __nv_bfloat16* p = static_cast<__nv_bfloat16*>(c.p);
      float pv = __bfloat162float(p[i]) * decay - step_size * m / denom;
      p[i] = __float2bfloat16(pv);
    } else {
      float* p = static_cast<float*>(c.p);
      p[i] = p[i] * decay - step_size * m / denom;
    }
  }
}

}  // namespace

void adamw_multi(const AdamWTensor* list, int count, float lr, float beta1, float beta2, float eps, float wd, int step,
                 cudaStream_t s) {
  const double bc1 = 1.0 - std::pow(static_cast<double>(beta1), step);
  const double bc2 = 1.0 - std::pow(static_cast<double>(beta2), step);
  Table tab;
  int nc = 0;
  auto flush = [&]() {
    if (nc == 0) return;
    adamw_kernel<<<nc, NT, 0, s>>>(tab, lr, beta1, beta2, eps, wd, static_cast<float>(bc1),
                                   static_cast<float>(std::sqrt(bc2)));
    check_cuda(cudaGetLastError(), "adamw");
    nc = 0;
  };
  for (int i = 0; i < count; ++i) {
    const AdamWTensor& t = list[i];
    const int esz_p = t.p_dtype ? 2 : 4, esz_g = t.g_dtype ? 2 : 4;
    for (int64_t off = 0; off < t.n; off += CHUNK) {
      Chunk& c = tab.c[nc];
      c.p = static_cast<char*>(t.p) + off * esz_p;
      c.g = static_cast<const char*>(t.g) + off * esz_g;
      c.m = t.m + off;
      c.v = t.v + off;
      c.n = static_cast<int>(t.n - off < CHUNK ? t.n - off : CHUNK);
      c.p_bf16 = static_cast<int8_t>(t.p_dtype);
      c.g_bf16 = static_cast<int8_t>(t.g_dtype);
      if (++nc == MAX_CHUNKS) flush();
    }
  }
  flush();
}

}  // namespace ttb
