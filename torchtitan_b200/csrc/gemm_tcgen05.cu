// Dense bf16 GEMM for sm_100a on the 5th-generation tensor cores.
//
//   D[M,N] (bf16) = sum_k A(m,k) * B(n,k)   (fp32 accumulation in TMEM)
//
// A is K-major ([M,K] row-major) or M-major ([K,M] row-major); B likewise
// ([N,K] or [K,N]).  This covers forward, dgrad and wgrad of a linear layer
// without any transpose copies.
//
// Design: persistent kernel, one CTA per SM (grid = min(tiles, #SMs)), tile
// 128x256x64, 4-stage TMA ring (48 KB/stage, 128-byte swizzle), warp roles:
//   warp 0      TMA producer (one elected thread)
//   warp 1      TMEM allocator + tcgen05.mma issuer (one elected thread)
//   warps 2..5  epilogue: tcgen05.ld TMEM -> registers -> bf16 -> global
// Two TMEM accumulators (2 x 256 fp32 columns = all 512 columns) let the
// epilogue of tile i overlap the main loop of tile i+1.  Tiles are visited in
// GROUP_M-row bands so consecutive CTAs share A/B panels in L2.
// All barrier waits are bounded (see sm100_ptx.cuh); a timeout sets
// gemm_error_code() and the kernel exits after releasing TMEM.
#include <cstdlib>
#include <stdexcept>
#include <string>

#include "launch_api.h"
#include "sm100_ptx.cuh"
#include "tma_host.h"

namespace ttb {
namespace gemm_impl {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;
constexpr int B_BYTES = BN * BK * 2;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024;
constexpr int NUM_THREADS = 192;
constexpr int GROUP_M = 8;
constexpr int TMEM_COLS = 512;

__device__ int g_err;

struct Params {
  int M, N, K;
  int num_m, num_n, num_k;
  __nv_bfloat16* D;
  int ldd;
  // grouped modes (0 = plain GEMM)
  //  1: per-M-tile group id tile_group[tm] (-1 = skip) selects B rows [g*b_group_rows, ...)
  //  2: group g = tile / (num_m*num_n) reduces over K rows [kstart[g], kstart[g]+klen[g]) and
  //     writes D + g*d_group_stride (klen = 0 writes zeros)
  int mode;
  int num_groups;
  const int* tile_group;
  const int* group_kstart;
  const int* group_klen;
  int b_group_rows;
  long long d_group_stride;
};

struct TileInfo {
  int tm, tn, g, k_base, nk;
  bool valid;
};

__device__ __forceinline__ void tile_coords(int t, const Params& p, int& tm, int& tn);

__device__ __forceinline__ int total_tiles(const Params& p) {
  return p.num_m * p.num_n * (p.mode == 2 ? p.num_groups : 1);
}

__device__ __forceinline__ TileInfo tile_info(int t, const Params& p) {
  TileInfo ti;
  ti.g = 0;
  ti.k_base = 0;
  ti.nk = p.num_k;
  ti.valid = true;
  if (p.mode == 2) {
    const int per = p.num_m * p.num_n;
    ti.g = t / per;
    tile_coords(t - ti.g * per, p, ti.tm, ti.tn);
    ti.k_base = p.group_kstart[ti.g];
    ti.nk = (p.group_klen[ti.g] + 63) / 64;
  } else {
    tile_coords(t, p, ti.tm, ti.tn);
    if (p.mode == 1) {
      ti.g = p.tile_group[ti.tm];
      ti.valid = ti.g >= 0;
    }
  }
  return ti;
}

__device__ __forceinline__ void tile_coords(int t, const Params& p, int& tm, int& tn) {
  const int per_group = GROUP_M * p.num_n;
  const int g = t / per_group;
  const int first_m = g * GROUP_M;
  const int gs = min(p.num_m - first_m, GROUP_M);
  const int r = t - g * per_group;
  tm = first_m + r % gs;
  tn = r / gs;
}

struct Shared {
  uint64_t full[STAGES], empty[STAGES], tfull[2], tempty[2];
  uint32_t tmem_base;
  int abort_flag;
};

template <bool A_MN, bool B_MN>
__device__ __forceinline__ void run_producer(const CUtensorMap* tmA, const CUtensorMap* tmB, const Params& p,
                                             Shared& sh, uint8_t* sA, uint8_t* sB) {
  int stage = 0;
  uint32_t phase = 0;
  const int tiles = total_tiles(p);
  for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
    const TileInfo ti = tile_info(t, p);
    if (!ti.valid) continue;
    const int tm = ti.tm, tn = ti.tn;
    const int bgo = (p.mode == 1) ? ti.g * p.b_group_rows : 0;
    for (int kb = 0; kb < ti.nk; ++kb) {
      if (!mbar_wait(&sh.empty[stage], phase ^ 1, &sh.abort_flag, &g_err, 1)) return;
      mbar_arrive_expect_tx(&sh.full[stage], STAGE_BYTES);
      uint8_t* a = sA + stage * A_BYTES;
      uint8_t* b = sB + stage * B_BYTES;
      const int k0 = ti.k_base + kb * BK;
      if constexpr (!A_MN) {
        tma_load_2d(a, tmA, &sh.full[stage], k0, tm * BM);
      } else {
#pragma unroll
        for (int j = 0; j < BM / 64; ++j) tma_load_2d(a + j * 8192, tmA, &sh.full[stage], tm * BM + j * 64, k0);
      }
      if constexpr (!B_MN) {
        tma_load_2d(b, tmB, &sh.full[stage], k0, bgo + tn * BN);
      } else {
#pragma unroll
        for (int j = 0; j < BN / 64; ++j)
          tma_load_2d(b + j * 8192, tmB, &sh.full[stage], tn * BN + j * 64, bgo + k0);
      }
      if (++stage == STAGES) {
        stage = 0;
        phase ^= 1;
      }
    }
  }
  // drain: wait until the MMA side has consumed every stage we filled
  for (int s = 0; s < STAGES; ++s) {
    if (!mbar_wait(&sh.empty[stage], phase ^ 1, &sh.abort_flag, &g_err, 2)) return;
    if (++stage == STAGES) {
      stage = 0;
      phase ^= 1;
    }
  }
}

template <bool A_MN, bool B_MN>
__device__ __forceinline__ void run_mma(const Params& p, Shared& sh, uint8_t* sA, uint8_t* sB) {
  constexpr uint32_t idesc = umma_idesc_bf16(BM, BN, A_MN, B_MN);
  int stage = 0;
  uint32_t phase = 0;
  int it = 0;
  const int tiles = total_tiles(p);
  for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
    const TileInfo ti = tile_info(t, p);
    if (!ti.valid || ti.nk == 0) continue;  // the epilogue skips / zero-fills these too
    const int acc = it & 1;
    const uint32_t acc_phase = (it >> 1) & 1;
    ++it;
    if (!mbar_wait(&sh.tempty[acc], acc_phase ^ 1, &sh.abort_flag, &g_err, 3)) return;
    tc_fence_after();
    const uint32_t d_tmem = sh.tmem_base + acc * BN;
    for (int kb = 0; kb < ti.nk; ++kb) {
      if (!mbar_wait(&sh.full[stage], phase, &sh.abort_flag, &g_err, 4)) return;
      tc_fence_after();
      const uint32_t a_addr = smem_u32(sA + stage * A_BYTES);
      const uint32_t b_addr = smem_u32(sB + stage * B_BYTES);
#pragma unroll
      for (int k = 0; k < BK / 16; ++k) {
        const uint64_t ad = A_MN ? umma_desc_sw128(a_addr + k * 2048, 8192, 1024) : umma_desc_sw128(a_addr + k * 32, 16, 1024);
        const uint64_t bd = B_MN ? umma_desc_sw128(b_addr + k * 2048, 8192, 1024) : umma_desc_sw128(b_addr + k * 32, 16, 1024);
        umma_bf16(d_tmem, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
      }
      umma_commit(&sh.empty[stage]);
      if (++stage == STAGES) {
        stage = 0;
        phase ^= 1;
      }
    }
    umma_commit(&sh.tfull[acc]);
  }
}

__device__ __forceinline__ void run_epilogue(const Params& p, Shared& sh, int warp, int lane) {
  const int q = warp & 3;  // TMEM lane quarter this warp may access
  int it = 0;
  const int tiles = total_tiles(p);
  const bool vec_ok = (p.ldd % 8) == 0;
  for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
    const TileInfo ti = tile_info(t, p);
    if (!ti.valid) continue;
    const int tm = ti.tm, tn = ti.tn;
    const int row = tm * BM + q * 32 + lane;
    __nv_bfloat16* dbase = p.D + (p.mode == 2 ? ti.g * p.d_group_stride : 0ll);
    __nv_bfloat16* drow = dbase + static_cast<size_t>(row) * p.ldd;
    if (ti.nk == 0) {  // empty group: its slice of D is zero
      if (row < p.M)
        for (int col = tn * BN; col < min(p.N, tn * BN + BN); ++col) drow[col] = __float2bfloat16(0.f);
      continue;
    }
    const int acc = it & 1;
    const uint32_t acc_phase = (it >> 1) & 1;
    ++it;
    if (!mbar_wait(&sh.tfull[acc], acc_phase, &sh.abort_flag, &g_err, 5)) return;
    tc_fence_after();
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(sh.tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN + c * 32, r);
      tmem_ld_wait();
      const int col = tn * BN + c * 32;
      if (row < p.M && col < p.N) {
        if (vec_ok && col + 32 <= p.N) {
          uint4* dst = reinterpret_cast<uint4*>(drow + col);
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint4 o;
            o.x = pack_bf16x2(__uint_as_float(r[8 * v + 0]), __uint_as_float(r[8 * v + 1]));
            o.y = pack_bf16x2(__uint_as_float(r[8 * v + 2]), __uint_as_float(r[8 * v + 3]));
            o.z = pack_bf16x2(__uint_as_float(r[8 * v + 4]), __uint_as_float(r[8 * v + 5]));
            o.w = pack_bf16x2(__uint_as_float(r[8 * v + 6]), __uint_as_float(r[8 * v + 7]));
            dst[v] = o;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (col + j < p.N) drow[col + j] = __float2bfloat16(__uint_as_float(r[j]));
        }
      }
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&sh.tempty[acc]);
  }
}

template <bool A_MN, bool B_MN>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, Params p) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ Shared sh;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&sh.full[s], 1);
      mbar_init(&sh.empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&sh.tfull[a], 1);
      mbar_init(&sh.tempty[a], 4);
    }
    sh.abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) tmem_alloc(&sh.tmem_base, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  if (warp == 0) {
    if (lane == 0) run_producer<A_MN, B_MN>(&tmA, &tmB, p, sh, sA, sB);
  } else if (warp == 1) {
    if (lane == 0) run_mma<A_MN, B_MN>(p, sh, sA, sB);
  } else {
    run_epilogue(p, sh, warp, lane);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(sh.tmem_base, TMEM_COLS);
  }
}

template <bool A_MN, bool B_MN>
void launch(const CUtensorMap& ta, const CUtensorMap& tb, const Params& p, cudaStream_t stream) {
  static bool attr_set = false;
  auto* k = gemm_kernel<A_MN, B_MN>;
  if (!attr_set) {
    check_cuda(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES), "gemm smem attr");
    attr_set = true;
  }
  static int sms = 0;
  if (sms == 0) {
    int dev;
    check_cuda(cudaGetDevice(&dev), "gemm dev");
    sms = num_sms(dev);
  }
  const int tiles = p.num_m * p.num_n * (p.mode == 2 ? p.num_groups : 1);
  const int grid = tiles < sms ? tiles : sms;
  if (grid == 0) return;
  k<<<grid, NUM_THREADS, SMEM_BYTES, stream>>>(ta, tb, p);
  check_cuda(cudaGetLastError(), "gemm launch");
}

}  // namespace gemm_impl

void gemm_bf16(const void* A, const void* B, void* D, int64_t M, int64_t N, int64_t K, bool a_mn, bool b_mn,
               cudaStream_t stream) {
  using namespace gemm_impl;
  if (M == 0 || N == 0) return;
  if (K == 0) {
    check_cuda(cudaMemsetAsync(D, 0, static_cast<size_t>(M) * N * 2, stream), "gemm memset");
    return;
  }
  if (M >= (1ll << 31) || N >= (1ll << 31) || K >= (1ll << 31)) throw std::runtime_error("gemm: dims too large");
  if ((a_mn ? M : K) % 8 != 0 || (b_mn ? N : K) % 8 != 0)
    throw std::runtime_error("gemm: contiguous dimension of each operand must be a multiple of 8");
  // CTA-pair kernel for large tiles (measured faster except for very wide N)
  static const bool pair_enabled = [] {
    const char* e = std::getenv("TTB_GEMM_2SM");
    return !(e && e[0] == '0');
  }();
  if (pair_enabled && M >= 512 && N >= 256 && N <= 32768) {
    gemm_bf16_2sm(A, B, D, M, N, K, a_mn, b_mn, stream);
    return;
  }
  const CUtensorMap ta = a_mn ? make_tmap_bf16_2d(A, K, M, M, 64, 64) : make_tmap_bf16_2d(A, M, K, K, BM, 64);
  const CUtensorMap tb = b_mn ? make_tmap_bf16_2d(B, K, N, N, 64, 64) : make_tmap_bf16_2d(B, N, K, K, BN, 64);
  Params p;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.num_m = (int)((M + BM - 1) / BM);
  p.num_n = (int)((N + BN - 1) / BN);
  p.num_k = (int)((K + BK - 1) / BK);
  p.D = reinterpret_cast<__nv_bfloat16*>(D);
  p.ldd = (int)N;
  p.mode = 0;
  p.num_groups = 1;
  p.tile_group = p.group_kstart = p.group_klen = nullptr;
  p.b_group_rows = 0;
  p.d_group_stride = 0;
  if (!a_mn && !b_mn) launch<false, false>(ta, tb, p, stream);
  else if (!a_mn && b_mn) launch<false, true>(ta, tb, p, stream);
  else if (a_mn && !b_mn) launch<true, false>(ta, tb, p, stream);
  else launch<true, true>(ta, tb, p, stream);
}

void gemm_bf16_grouped(const void* A, const void* B, void* D, int64_t M, int64_t N, int64_t K, bool a_mn,
                       bool b_mn, int mode, int num_groups, const int* tile_group, const int* kstart,
                       const int* klen, int64_t b_total_rows, int b_group_rows, cudaStream_t stream) {
  using namespace gemm_impl;
  if (M == 0 || N == 0 || num_groups == 0) return;
  if ((a_mn ? M : K) % 8 != 0 || (b_mn ? N : K) % 8 != 0)
    throw std::runtime_error("grouped gemm: contiguous dimension of each operand must be a multiple of 8");
  // mode 1: A is [M, K] (or [K, M]) over all padded rows; B holds num_groups stacked matrices
  // mode 2: A is [Ktot, M], B is [Ktot, N] (both M/N-major); D is [num_groups, M, N]
  const CUtensorMap ta = a_mn ? make_tmap_bf16_2d(A, K, M, M, 64, 64) : make_tmap_bf16_2d(A, M, K, K, BM, 64);
  const CUtensorMap tb = b_mn ? make_tmap_bf16_2d(B, b_total_rows, N, N, 64, 64)
                              : make_tmap_bf16_2d(B, b_total_rows, K, K, BN, 64);
  Params p;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.num_m = (int)((M + BM - 1) / BM);
  p.num_n = (int)((N + BN - 1) / BN);
  p.num_k = (int)((K + BK - 1) / BK);
  p.D = reinterpret_cast<__nv_bfloat16*>(D);
  p.ldd = (int)N;
  p.mode = mode;
  p.num_groups = num_groups;
  p.tile_group = tile_group;
  p.group_kstart = kstart;
  p.group_klen = klen;
  p.b_group_rows = b_group_rows;
  p.d_group_stride = (long long)M * N;
  if (!a_mn && !b_mn) launch<false, false>(ta, tb, p, stream);
  else if (!a_mn && b_mn) launch<false, true>(ta, tb, p, stream);
  else if (a_mn && !b_mn) launch<true, false>(ta, tb, p, stream);
  else launch<true, true>(ta, tb, p, stream);
}

int gemm_error_code(bool reset) {
  int v = 0;
  check_cuda(cudaMemcpyFromSymbol(&v, gemm_impl::g_err, sizeof(int)), "gemm error read");
  if (reset) {
    int z = 0;
    check_cuda(cudaMemcpyToSymbol(gemm_impl::g_err, &z, sizeof(int)), "gemm error reset");
  }
  return v;
}

}  // namespace ttb
