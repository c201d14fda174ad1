// MXFP8 quantization for the block-scaled GEMM (gemm_mxfp8.cu).
//
// x [R, C] bf16 (C contiguous) -> codes [R, Cp] FP8 E4M3 (Cp = C rounded up to
// 128, zero padded) and E8M0 scale records in the tcgen05 blocked layout (see
// gemm_mxfp8.cu) for ceil(R/128)*128 rows.  One thread quantizes one group of 32
// consecutive elements of a row:
//   amax = max |x|;  e = ceil(log2(amax / 448))  (RCEIL, via frexp: exact)
//   code = e4m3_rne_satfinite(x * 2^-e);   scale byte = e + 127
// Padding groups get code 0 and scale byte 127 (2^0).
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <stdexcept>

#include "launch_api.h"

namespace ttb {
namespace mxq_impl {

__global__ void __launch_bounds__(256) mx_quant_kernel(const __nv_bfloat16* __restrict__ x, int64_t R, int64_t C,
                                                       int64_t ldx, uint8_t* __restrict__ codes, int64_t Cp,
                                                       uint8_t* __restrict__ sf, int64_t Rp) {
  const int64_t groups_per_row = Cp / 32;
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (gid >= Rp * groups_per_row) return;
  const int64_t r = gid / groups_per_row;
  const int64_t g = gid - r * groups_per_row;
  const int64_t c0 = g * 32;
  float v[32];
  const bool live = r < R && c0 < C;
  if (live && c0 + 32 <= C && (ldx % 8) == 0) {
    const uint4* src = reinterpret_cast<const uint4*>(x + r * ldx + c0);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 w = src[q];
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float2 f = __bfloat1622float2(h[u]);
        v[8 * q + 2 * u] = f.x;
        v[8 * q + 2 * u + 1] = f.y;
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = (live && c0 + i < C) ? __bfloat162float(x[r * ldx + c0 + i]) : 0.f;
  }
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
  int e;
  if (amax == 0.f) {
    e = -127;
  } else {
    int p;
    const float m = frexpf(amax / 448.f, &p);  // amax/448 = m * 2^p, m in [0.5, 1)
    e = (m == 0.5f) ? p - 1 : p;               // ceil(log2(amax / 448)), exactly
    e = max(-127, min(127, e));
  }
  if (!live) e = 0;
  uint32_t packed[8];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float a = ldexpf(v[2 * i], -e), b = ldexpf(v[2 * i + 1], -e);
    const __nv_fp8x2_storage_t two = __nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
    if (i % 2 == 0) packed[i / 2] = two;
    else packed[i / 2] |= static_cast<uint32_t>(two) << 16;
  }
  uint4* dst = reinterpret_cast<uint4*>(codes + r * Cp + c0);
  if (r < R) {
    dst[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    dst[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
  }
  // blocked scale layout: record (r/128, g/4), byte (r%32)*16 + ((r%128)/32)*4 + g%4
  const int64_t nkb = Cp / 128;
  const int64_t rec = (r / 128) * nkb + g / 4;
  const int rin = static_cast<int>(r % 128);
  sf[rec * 512 + (rin % 32) * 16 + (rin / 32) * 4 + (g % 4)] = static_cast<uint8_t>(e + 127);
}

}  // namespace mxq_impl

void mx_quantize(const void* x, int64_t R, int64_t C, int64_t ldx, void* codes, void* sf, cudaStream_t s) {
  using namespace mxq_impl;
  const int64_t Cp = (C + 127) / 128 * 128;
  const int64_t Rp = (R + 127) / 128 * 128;
  const int64_t n = Rp * (Cp / 32);
  if (n == 0) return;
  mx_quant_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), R, C, ldx,
                                                               static_cast<uint8_t*>(codes), Cp,
                                                               static_cast<uint8_t*>(sf), Rp);
  check_cuda(cudaGetLastError(), "mx quantize launch");
}

}  // namespace ttb
