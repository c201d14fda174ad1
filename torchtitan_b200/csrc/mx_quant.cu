// MXFP8 quantization for the block-scaled GEMM (gemm_mxfp8.cu).
//
// x [R, C] bf16 (C contiguous) -> codes [R, Cp] FP8 E4M3 (Cp = C rounded up to
// 128, zero padded) and E8M0 scale records in the tcgen05 blocked layout (see
// gemm_mxfp8.cu) for ceil(R/128)*128 rows.  Every group of 32 consecutive elements of a
// row is quantized as:
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

// One CTA per (128-row block, 128-column block): thread t quantizes row 128*rb + t over the 128
// columns, i.e. the four 32-element groups whose scales form one 32-bit word of the record, so
// the record is written as 128 aligned 4-byte stores and each thread's codes are one 128-byte
// line. All 16 of a thread's 16-byte loads are issued before the first group is converted.
__device__ __forceinline__ float pow2i(int n) {  // 2^n for -126 <= n <= 127, exact
  return __int_as_float((n + 127) << 23);
}

__device__ __forceinline__ int mx_exponent(float amax) {
  if (amax == 0.f) return -127;
  int p;
  const float m = frexpf(amax / 448.f, &p);  // amax/448 = m * 2^p, m in [0.5, 1)
  const int e = (m == 0.5f) ? p - 1 : p;     // ceil(log2(amax / 448)), exactly
  return max(-127, min(127, e));
}

__global__ void __launch_bounds__(128) mx_quant_kernel(const __nv_bfloat16* __restrict__ x, int64_t R, int64_t C,
                                                       int64_t ldx, uint8_t* __restrict__ codes, int64_t Cp,
                                                       uint8_t* __restrict__ sf) {
  const int64_t rb = blockIdx.y, kb = blockIdx.x, nkb = gridDim.x;
  const int t = threadIdx.x;
  const int64_t r = rb * 128 + t;
  const int64_t c0 = kb * 128;
  const bool row_live = r < R;
  uint4 raw[16];
  const bool vec = row_live && c0 + 128 <= C && (ldx % 8) == 0;
  if (vec) {
    const uint4* src = reinterpret_cast<const uint4*>(x + r * ldx + c0);
#pragma unroll
    for (int q = 0; q < 16; ++q) raw[q] = src[q];
  }
  uint32_t sfw = 0;
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    float v[32];
    if (vec) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw[4 * g + q]);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float2 f = __bfloat1622float2(h[u]);
          v[8 * q + 2 * u] = f.x;
          v[8 * q + 2 * u + 1] = f.y;
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int64_t c = c0 + 32 * g + i;
        v[i] = (row_live && c < C) ? __bfloat162float(x[r * ldx + c]) : 0.f;
      }
    }
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
    // groups wholly in the row or column padding get scale 2^0
    const bool live = row_live && c0 + 32 * g < C;
    const int e = live ? mx_exponent(amax) : 0;
    sfw |= static_cast<uint32_t>(e + 127) << (8 * g);
    if (row_live) {
      const float inv = pow2i(-e);  // e in [-127, 120] for finite bf16 input: -e is in range
      uint32_t packed[8];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const __nv_fp8x2_storage_t two =
            __nv_cvt_float2_to_fp8x2(make_float2(v[2 * i] * inv, v[2 * i + 1] * inv), __NV_SATFINITE, __NV_E4M3);
        if (i % 2 == 0) packed[i / 2] = two;
        else packed[i / 2] |= static_cast<uint32_t>(two) << 16;
      }
      uint4* dst = reinterpret_cast<uint4*>(codes + r * Cp + c0 + 32 * g);
      dst[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
      dst[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
    }
  }
  // blocked scale layout: record (rb, kb), word at byte (t%32)*16 + (t/32)*4
  *reinterpret_cast<uint32_t*>(sf + (rb * nkb + kb) * 512 + (t % 32) * 16 + (t / 32) * 4) = sfw;
}

// ---- Float8 (E4M3) with one fp32 scale per row or per tensor --------------------------------
// scale = 448 / max(amax, 1e-12); code = cvt.rn.satfinite.e4m3(x * scale); inv = 1 / scale. Codes
// are [R, Cp] with the columns zero padded to a multiple of 128 (the GEMM's K step). Measured on
// a B200: the conversion instruction rounds a product within a few fp32 ulps of an E4M3 tie as
// the tie (about 0.1 % of codes one E4M3 step from the correctly rounded value); the MX codes are
// exact because their scales are powers of two.
__device__ __forceinline__ float f8_scale(float amax) { return __fdiv_rn(448.f, fmaxf(amax, 1e-12f)); }

__device__ __forceinline__ uint2 f8_codes8(const float (&v)[8], float scale) {
  uint32_t w[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const __nv_fp8x2_storage_t lo = __nv_cvt_float2_to_fp8x2(make_float2(v[4 * h] * scale, v[4 * h + 1] * scale),
                                                             __NV_SATFINITE, __NV_E4M3);
    const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(
        make_float2(v[4 * h + 2] * scale, v[4 * h + 3] * scale), __NV_SATFINITE, __NV_E4M3);
    w[h] = static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
  }
  return make_uint2(w[0], w[1]);
}

// 8 elements of row r starting at column c (zeros past C)
__device__ __forceinline__ void load8_row(const __nv_bfloat16* x, int64_t r, int64_t c, int64_t C, int64_t ldx,
                                          bool vec, float (&v)[8]) {
  if (vec && c + 8 <= C) {
    const uint4 w = *reinterpret_cast<const uint4*>(x + r * ldx + c);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float2 f = __bfloat1622float2(h[u]);
      v[2 * u] = f.x;
      v[2 * u + 1] = f.y;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = c + i < C ? __bfloat162float(x[r * ldx + c + i]) : 0.f;
  }
}

// rowwise: one warp per row, amax pass then a second (L2-resident) pass writing the codes
__global__ void __launch_bounds__(256) f8_rowwise_kernel(const __nv_bfloat16* __restrict__ x, int64_t R, int64_t C,
                                                         int64_t ldx, uint8_t* __restrict__ codes, int64_t Cp,
                                                         float* __restrict__ inv) {
  const int64_t r = static_cast<int64_t>(blockIdx.x) * 8 + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (r >= R) return;
  const bool vec = (ldx % 8) == 0;
  float amax = 0.f;
  for (int64_t c = lane * 8; c < C; c += 256) {
    float v[8];
    load8_row(x, r, c, C, ldx, vec, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float scale = f8_scale(amax);
  if (lane == 0) inv[r] = __frcp_rn(scale);
  for (int64_t c = lane * 8; c < Cp; c += 256) {
    float v[8];
    load8_row(x, r, c, C, ldx, vec, v);
    *reinterpret_cast<uint2*>(codes + r * Cp + c) = f8_codes8(v, scale);
  }
}

// tensorwise: grid-stride amax into one word (non-negative floats order like their bit patterns)
__global__ void __launch_bounds__(256) f8_amax_kernel(const __nv_bfloat16* __restrict__ x, int64_t R, int64_t C,
                                                      int64_t ldx, unsigned int* __restrict__ amax_word) {
  const int64_t per_row = (C + 7) / 8;
  const bool vec = (ldx % 8) == 0;
  float amax = 0.f;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < R * per_row;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / per_row, c = (i - r * per_row) * 8;
    float v[8];
    load8_row(x, r, c, C, ldx, vec, v);
#pragma unroll
    for (int k = 0; k < 8; ++k) amax = fmaxf(amax, fabsf(v[k]));
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) atomicMax(amax_word, __float_as_uint(amax));
}

__global__ void __launch_bounds__(256) f8_tensorwise_kernel(const __nv_bfloat16* __restrict__ x, int64_t R,
                                                            int64_t C, int64_t ldx, uint8_t* __restrict__ codes,
                                                            int64_t Cp, const unsigned int* __restrict__ amax_word,
                                                            float* __restrict__ inv) {
  const float scale = f8_scale(__uint_as_float(*amax_word));
  if (blockIdx.x == 0 && threadIdx.x == 0) inv[0] = __frcp_rn(scale);
  const int64_t per_row = Cp / 8;
  const bool vec = (ldx % 8) == 0;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < R * per_row;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / per_row, c = (i - r * per_row) * 8;
    float v[8];
    load8_row(x, r, c, C, ldx, vec, v);
    *reinterpret_cast<uint2*>(codes + r * Cp + c) = f8_codes8(v, scale);
  }
}

}  // namespace mxq_impl

void mx_quantize(const void* x, int64_t R, int64_t C, int64_t ldx, void* codes, void* sf, cudaStream_t s) {
  using namespace mxq_impl;
  const int64_t Cp = (C + 127) / 128 * 128;
  const int64_t Rp = (R + 127) / 128 * 128;
  if (Rp == 0 || Cp == 0) return;
  if (Rp / 128 > 65535) throw std::runtime_error("mx quantize: too many rows");
  const dim3 grid(static_cast<unsigned>(Cp / 128), static_cast<unsigned>(Rp / 128));
  mx_quant_kernel<<<grid, 128, 0, s>>>(static_cast<const __nv_bfloat16*>(x), R, C, ldx, static_cast<uint8_t*>(codes),
                                        Cp, static_cast<uint8_t*>(sf));
  check_cuda(cudaGetLastError(), "mx quantize launch");
}

void f8_quantize(const void* x, int64_t R, int64_t C, int64_t ldx, bool rowwise, void* codes, float* inv,
                 unsigned int* amax_word, cudaStream_t s) {
  using namespace mxq_impl;
  const int64_t Cp = (C + 127) / 128 * 128;
  if (R == 0 || C == 0) return;
  const auto* xb = static_cast<const __nv_bfloat16*>(x);
  auto* cb = static_cast<uint8_t*>(codes);
  if (rowwise) {
    f8_rowwise_kernel<<<static_cast<unsigned>((R + 7) / 8), 256, 0, s>>>(xb, R, C, ldx, cb, Cp, inv);
  } else {
    int dev = 0;
    check_cuda(cudaGetDevice(&dev), "f8 quantize device");
    const unsigned grid = static_cast<unsigned>(num_sms(dev) * 8);
    check_cuda(cudaMemsetAsync(amax_word, 0, sizeof(unsigned int), s), "f8 amax reset");
    f8_amax_kernel<<<grid, 256, 0, s>>>(xb, R, C, ldx, amax_word);
    f8_tensorwise_kernel<<<grid, 256, 0, s>>>(xb, R, C, ldx, cb, Cp, amax_word, inv);
  }
  check_cuda(cudaGetLastError(), "f8 quantize launch");
}

}  // namespace ttb
