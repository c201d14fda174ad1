// Dense bf16 GEMM on CTA pairs (tcgen05 cta_group::2), 256x256x64 tiles.
//
//   D[M,N] = sum_k A(m,k) B(n,k)     (A, B K-major or M/N-major as in gemm_tcgen05.cu)
//
// A cluster of two CTAs on two SMs computes one 256x256 tile: CTA r loads
// rows [128r, 128r+128) of the A tile and rows [128r, 128r+128) of the B
// tile (N direction) into its own shared memory, so each SM streams half of
// B instead of all of it.  TMA loads carry .cta_group::2 and complete on the
// leader CTA's barrier.  Only the leader's MMA thread issues
// tcgen05.mma.cta_group::2 (M=256, N=256); the accumulator of rows owned by
// CTA r lands in CTA r's TMEM (2 x 256 fp32 columns, double-buffered).
// Commits are multicast to both CTAs' barriers; each CTA's epilogue drains
// its own TMEM lanes and arrives on the leader's accumulator-empty barrier.
// No TMA load uses multicast.  Every wait is bounded (sm100_ptx.cuh).
#include <stdexcept>

#include "launch_api.h"
#include "sm100_ptx.cuh"
#include "tma_host.h"

namespace ttb {
namespace gemm2 {

constexpr int BMH = 128;  // rows per CTA (pair tile = 256)
constexpr int BN = 256;   // pair tile width; each CTA holds 128 rows of B
constexpr int BNH = 128;
constexpr int BK = 64, STAGES = 6;
constexpr int A_BYTES = BMH * BK * 2;
constexpr int B_BYTES = BNH * BK * 2;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024;
constexpr int NUM_THREADS = 192;
constexpr int GROUP_M = 8;
constexpr uint32_t PEER_MASK = 0xFEFFFFFFu;  // clears the CTA-in-pair bit of a shared::cluster address

__device__ int g_err;

struct Params {
  int M, N, K;
  int num_m, num_n, num_k;  // num_m counts 256-row pair tiles
  __nv_bfloat16* D;
  int ldd;
};

struct Shared {
  uint64_t full[STAGES], empty[STAGES], tfull[2], tempty[2];
  uint32_t tmem_base;
  int abort_flag;
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* m, uint64_t* bar, int x, int y) {
  const uint32_t mbar = smem_u32(bar) & PEER_MASK;  // leader CTA's barrier
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::
          "r"(smem_u32(dst)),
      "l"(m), "r"(mbar), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void umma_bf16_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// arrive on the barrier at the same offset in both CTAs of the pair when prior MMAs finish
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"((uint16_t)0x3)
      : "memory");
}

__device__ __forceinline__ void arrive_on_leader(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b32 ra;\n\t"
      "mapa.shared::cluster.u32 ra, %0, 0;\n\t"
      "mbarrier.arrive.release.cluster.shared::cluster.b64 _, [ra];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
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

template <bool A_MN, bool B_MN>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, Params p) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ Shared sh;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int cluster = blockIdx.x / 2, nclusters = gridDim.x / 2;
  const int tiles = p.num_m * p.num_n;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&sh.full[s], 1);
      mbar_init(&sh.empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&sh.tfull[a], 1);
      mbar_init(&sh.tempty[a], 8);  // 4 epilogue warps x 2 CTAs
    }
    sh.abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&sh.tmem_base)),
                 "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = cluster; ok && t < tiles; t += nclusters) {
        int tm, tn;
        tile_coords(t, p, tm, tn);
        const int m0 = tm * 2 * BMH + rank * BMH, n0 = tn * BN + rank * BNH;
        for (int kb = 0; kb < p.num_k; ++kb) {
          if (!mbar_wait(&sh.empty[stage], phase ^ 1, &sh.abort_flag, &g_err, 61)) { ok = false; break; }
          if (leader) mbar_arrive_expect_tx(&sh.full[stage], 2 * STAGE_BYTES);
          uint8_t* a = sA + stage * A_BYTES;
          uint8_t* b = sB + stage * B_BYTES;
          const int k0 = kb * BK;
          if constexpr (!A_MN) {
            tma_load_2d_pair(a, &tmA, &sh.full[stage], k0, m0);
          } else {
#pragma unroll
            for (int j = 0; j < BMH / 64; ++j) tma_load_2d_pair(a + j * 8192, &tmA, &sh.full[stage], m0 + j * 64, k0);
          }
          if constexpr (!B_MN) {
            tma_load_2d_pair(b, &tmB, &sh.full[stage], k0, n0);
          } else {
#pragma unroll
            for (int j = 0; j < BNH / 64; ++j) tma_load_2d_pair(b + j * 8192, &tmB, &sh.full[stage], n0 + j * 64, k0);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // drain: every filled stage has been consumed by the pair's MMAs
      for (int s = 0; ok && s < STAGES; ++s) {
        if (!mbar_wait(&sh.empty[stage], phase ^ 1, &sh.abort_flag, &g_err, 62)) break;
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = umma_idesc_bf16(2 * BMH, BN, A_MN, B_MN);
      int stage = 0, it = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = cluster; ok && t < tiles; t += nclusters, ++it) {
        const int acc = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        if (!mbar_wait(&sh.tempty[acc], acc_phase ^ 1, &sh.abort_flag, &g_err, 63)) break;
        tc_fence_after();
        const uint32_t d_tmem = sh.tmem_base + acc * BN;
        for (int kb = 0; kb < p.num_k; ++kb) {
          if (!mbar_wait(&sh.full[stage], phase, &sh.abort_flag, &g_err, 64)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * A_BYTES);
          const uint32_t b_addr = smem_u32(sB + stage * B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = A_MN ? umma_desc_sw128(a_addr + k * 2048, 8192, 1024)
                                     : umma_desc_sw128(a_addr + k * 32, 16, 1024);
            const uint64_t bd = B_MN ? umma_desc_sw128(b_addr + k * 2048, 8192, 1024)
                                     : umma_desc_sw128(b_addr + k * 32, 16, 1024);
            umma_bf16_pair(d_tmem, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit_pair(&sh.empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (ok) umma_commit_pair(&sh.tfull[acc]);
      }
    }
  } else {
    const int q = warp & 3;
    const bool vec_ok = (p.ldd % 8) == 0;
    int it = 0;
    for (int t = cluster; t < tiles; t += nclusters, ++it) {
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      int tm, tn;
      tile_coords(t, p, tm, tn);
      if (!mbar_wait(&sh.tfull[acc], acc_phase, &sh.abort_flag, &g_err, 65)) break;
      tc_fence_after();
      const int row = tm * 2 * BMH + rank * BMH + q * 32 + lane;
      __nv_bfloat16* drow = p.D + static_cast<size_t>(row) * p.ldd;
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
      if (lane == 0) arrive_on_leader(&sh.tempty[acc]);
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the peer's remote arrivals and the pair MMAs are done before TMEM is released
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(sh.tmem_base), "r"(512) : "memory");
  }
}

template <bool A_MN, bool B_MN>
void launch(const CUtensorMap& ta, const CUtensorMap& tb, const Params& p, cudaStream_t stream) {
  static bool attr_set = false;
  auto* k = gemm2_kernel<A_MN, B_MN>;
  if (!attr_set) {
    check_cuda(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES), "gemm2 smem attr");
    attr_set = true;
  }
  int dev;
  check_cuda(cudaGetDevice(&dev), "gemm2 dev");
  const int sms = num_sms(dev);
  const int tiles = p.num_m * p.num_n;
  const int clusters = tiles < sms / 2 ? tiles : sms / 2;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * clusters, 1, 1);
  cfg.blockDim = dim3(NUM_THREADS, 1, 1);
  cfg.dynamicSmemBytes = SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  check_cuda(cudaLaunchKernelEx(&cfg, k, ta, tb, p), "gemm2 launch");
}

}  // namespace gemm2

void gemm_bf16_2sm(const void* A, const void* B, void* D, int64_t M, int64_t N, int64_t K, bool a_mn, bool b_mn,
                   cudaStream_t stream) {
  using namespace gemm2;
  const CUtensorMap ta = a_mn ? make_tmap_bf16_2d(A, K, M, M, 64, 64) : make_tmap_bf16_2d(A, M, K, K, BMH, 64);
  const CUtensorMap tb = b_mn ? make_tmap_bf16_2d(B, K, N, N, 64, 64) : make_tmap_bf16_2d(B, N, K, K, BNH, 64);
  Params p;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.num_m = (int)((M + 2 * BMH - 1) / (2 * BMH));
  p.num_n = (int)((N + BN - 1) / BN);
  p.num_k = (int)((K + BK - 1) / BK);
  p.D = reinterpret_cast<__nv_bfloat16*>(D);
  p.ldd = (int)N;
  if (!a_mn && !b_mn) launch<false, false>(ta, tb, p, stream);
  else if (!a_mn && b_mn) launch<false, true>(ta, tb, p, stream);
  else if (a_mn && !b_mn) launch<true, false>(ta, tb, p, stream);
  else launch<true, true>(ta, tb, p, stream);
}

int gemm2_error_code(bool reset) {
  int v = 0;
  check_cuda(cudaMemcpyFromSymbol(&v, gemm2::g_err, sizeof(int)), "gemm2 error read");
  if (reset) {
    int z = 0;
    check_cuda(cudaMemcpyToSymbol(gemm2::g_err, &z, sizeof(int)), "gemm2 error reset");
  }
  return v;
}

}  // namespace ttb
