// MXFP8 block-scaled GEMM for sm_100a (tcgen05.mma kind::mxf8f6f4.block_scale).
//
//   D[M,N] (bf16) = sum_k A(m,k) * 2^(sa(m,k/32)-127) * B(n,k) * 2^(sb(n,k/32)-127)
//
// A [M,K] and B [N,K] are FP8 E4M3 codes, K contiguous (every GEMM of the MX
// training recipe -- forward, dgrad, wgrad -- is given operands quantized
// along its contraction dimension, so both are always K-major).  The E8M0
// scale factors use the tcgen05 "blocked" layout: for every 128-row block mb
// and every 128-element K block kb a 512-byte record at (mb * nKB + kb) * 512
// holds, at byte m0 * 16 + m1 * 4 + j, the scale of row mb*128 + 32*m1 + m0
// for the j-th 32-element group -- i.e. each 32-bit word holds the four
// scales one row needs for 128 K, which is the TMEM word the MMA reads.
//
// Two tile shapes, one template:
//   BN = 128: 128x128x128 tiles, 6-stage ring, two 128-column accumulators (the epilogue of
//             tile i overlaps the MMAs of tile i+1), 4 epilogue warps.
//   BN = 256: 128x256x128 tiles, 4-stage ring, one 256-column accumulator (the other half of
//             TMEM holds the scale records). Eight epilogue warps (two per TMEM lane quadrant,
//             128 columns each) copy the whole accumulator into registers and release it at
//             once, so the next tile's MMAs wait only for the TMEM reads; the bf16 conversion
//             and the global stores overlap them. Per MMA of K = 32 the tensor core reads
//             4 KB of A and 8 KB of B from shared memory for 2*128*256*32 FLOPs, twice the
//             work per byte of the 128-wide tile, which the shared-memory bandwidth bounds.
//   warp 0      producer: TMA for the A/B tiles (128-byte swizzle) and 512-byte bulk copies
//               of the scale records (one for A, BN/128 for B), one mbarrier per stage
//   warp 1      TMEM allocator + MMA issuer: per stage, tcgen05.cp of the scale records into
//               TMEM (32x128b, broadcast to the 4 lane quadrants; B's second record four
//               columns after the first), then 4 MMAs of K=32 selecting scale byte j
//   warps 2..   epilogue: TMEM -> registers -> bf16 -> global
// Grouped rows (routed experts): B is the stack of num_groups [N, K] matrices and M-tile tm
// multiplies group tile_group[tm] (N a multiple of 128, so every group starts on a scale-record
// block); tiles whose group is negative are skipped by all three roles alike.
// Every wait is bounded; a timeout sets mxgemm_error_code() and the kernel
// returns after releasing TMEM.  K must be a multiple of 128 (callers pad).
#include <stdexcept>

#include "launch_api.h"
#include "sm100_ptx.cuh"
#include "tma_host.h"

namespace ttb {
namespace mx_impl {

constexpr int BM = 128, BK = 128;
constexpr int A_BYTES = BM * BK;  // fp8
constexpr int SF_BYTES = 512;     // one blocked scale record
constexpr int GROUP_M = 8;
constexpr int TMEM_COLS = 512;

template <int BN>
struct Cfg {
  static constexpr int STAGES = BN == 256 ? 4 : 6;
  static constexpr int ACC_STAGES = BN == 256 ? 1 : 2;
  static constexpr int EPI_WARPS = BN == 256 ? 8 : 4;
  static constexpr int NUM_THREADS = 64 + 32 * EPI_WARPS;
  static constexpr int B_BYTES = BN * BK;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int SF_STAGE = SF_BYTES * (1 + BN / 128);  // A record + B records
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + STAGES * SF_STAGE + 1024;
  static constexpr int ACC_COLS = BN;                          // fp32 accumulator columns per tile
  static constexpr int SF_COL0 = ACC_STAGES * ACC_COLS;        // scale records after the accumulators
  static constexpr int SF_COLS_PER_STAGE = 4 + 4 * (BN / 128);
  static_assert(SF_COL0 + STAGES * SF_COLS_PER_STAGE <= TMEM_COLS, "TMEM budget");
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
};

__device__ int g_err;

struct Params {
  int M, N, K;
  int b_records;  // 128-row scale-record blocks of B (rows rounded up to 128)
  int num_m, num_n, num_k;
  const uint8_t* sfa;  // blocked scale records of A
  const uint8_t* sfb;
  __nv_bfloat16* D;
  int ldd;
  int sf_unit;          // scale records are all 2^0: every stage copies the one unit record
  const float* sa;      // optional output scales: D[m, n] *= sa[m or 0] * sb[n or 0]
  const float* sb;
  int sa_rows, sb_rows;  // 1: one scale per row of A / of B; 0: one scale for the operand
  const int* tile_group;  // grouped rows: B group of each M-tile (nullptr: group 0 everywhere)
};

__device__ __forceinline__ int tile_group_of(const Params& p, int tm) { return p.tile_group ? p.tile_group[tm] : 0; }

__device__ __align__(128) uint8_t g_unit_sf[SF_BYTES];  // E8M0 127 (= 2^0) bytes, set on first use

struct Shared {
  uint64_t full[6], empty[6], tfull[2], tempty[2];
  uint32_t tmem_base;
  int abort_flag;
};

__device__ __forceinline__ void tile_coords(int t, const Params& p, int& tm, int& tn) {  // grouped raster
  const int per_group = GROUP_M * p.num_n;
  const int g = t / per_group;
  const int first_m = g * GROUP_M;
  const int gs = min(p.num_m - first_m, GROUP_M);
  const int r = t - g * per_group;
  tm = first_m + r % gs;
  tn = r / gs;
}

// 1-D bulk copy global -> shared, completing on an mbarrier (no multicast)
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Shared-memory descriptor without swizzle for the tcgen05.cp source: 32 rows of
// 16 bytes = four 8x16-byte core matrices 128 bytes apart.
__device__ __forceinline__ uint64_t sf_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(512u >> 4) << 16;  // leading (K) offset: a single core-matrix column
  d |= static_cast<uint64_t>(128u >> 4) << 32;  // stride between 8-row core matrices
  d |= static_cast<uint64_t>(1) << 46;          // descriptor version for sm100
  return d;                                     // layout type 0 = no swizzle
}

// 32 lanes x 128 bits from shared memory into TMEM, replicated to all four lane quadrants
__device__ __forceinline__ void tmem_cp_32x128b_x4(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// Instruction descriptor, kind::mxf8f6f4 with E4M3 A/B, E8M0 scales, K-major A and B
__host__ __device__ constexpr uint32_t idesc_mx(int M, int N, int a_sf_id, int b_sf_id) {
  return (static_cast<uint32_t>(b_sf_id & 3) << 4) |   // B scale byte
         (0u << 7) | (0u << 10) |                       // A, B format E4M3
         (static_cast<uint32_t>(N >> 3) << 17) |        // N
         (1u << 23) |                                   // scale format E8M0
         (static_cast<uint32_t>(M >> 4) << 24) |        // M
         (static_cast<uint32_t>(a_sf_id & 3) << 29);    // A scale byte
}

__device__ __forceinline__ void umma_mx(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t tsfa, uint32_t tsfb, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(tsfa), "r"(tsfb));
}

template <int BN>
__device__ __forceinline__ void run_producer(const CUtensorMap* tmA, const CUtensorMap* tmB, const Params& p,
                                             Shared& sh, uint8_t* sA, uint8_t* sB, uint8_t* sSF) {
  using C = Cfg<BN>;
  int stage = 0;
  uint32_t phase = 0;
  const int tiles = p.num_m * p.num_n;
  for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
    int tm, tn;
    tile_coords(t, p, tm, tn);
    const int g = tile_group_of(p, tm);
    if (g < 0) continue;
    // B's scale records of this tile: 128-row blocks tn*BN/128 .. of group g; blocks past the
    // group's padded rows are not copied (their TMEM columns only scale output columns >= N)
    const int rb0 = g * p.b_records + tn * (BN / 128);
    const int nrec = min(BN / 128, p.b_records - tn * (BN / 128));
    for (int kb = 0; kb < p.num_k; ++kb) {
      if (!mbar_wait(&sh.empty[stage], phase ^ 1, &sh.abort_flag, &g_err, 1)) return;
      mbar_arrive_expect_tx(&sh.full[stage], C::STAGE_BYTES + (1 + nrec) * SF_BYTES);
      tma_load_2d(sA + stage * A_BYTES, tmA, &sh.full[stage], kb * BK, tm * BM);
      tma_load_2d(sB + stage * C::B_BYTES, tmB, &sh.full[stage], kb * BK, g * p.N + tn * BN);
      uint8_t* sf = sSF + stage * C::SF_STAGE;
      const size_t ua = p.sf_unit ? 0 : 1;  // unit records: always record 0 of the unit buffer
      bulk_load(sf, p.sfa + ua * (static_cast<size_t>(tm) * p.num_k + kb) * SF_BYTES, SF_BYTES, &sh.full[stage]);
      for (int r = 0; r < nrec; ++r)
        bulk_load(sf + (1 + r) * SF_BYTES, p.sfb + ua * (static_cast<size_t>(rb0 + r) * p.num_k + kb) * SF_BYTES,
                  SF_BYTES, &sh.full[stage]);
      if (++stage == C::STAGES) {
        stage = 0;
        phase ^= 1;
      }
    }
  }
  for (int s = 0; s < C::STAGES; ++s) {  // drain: every filled stage consumed
    if (!mbar_wait(&sh.empty[stage], phase ^ 1, &sh.abort_flag, &g_err, 2)) return;
    if (++stage == C::STAGES) {
      stage = 0;
      phase ^= 1;
    }
  }
}

template <int BN>
__device__ __forceinline__ void run_mma(const Params& p, Shared& sh, uint8_t* sA, uint8_t* sB, uint8_t* sSF) {
  using C = Cfg<BN>;
  int stage = 0;
  uint32_t phase = 0;
  int it = 0;
  const int tiles = p.num_m * p.num_n;
  for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
    if (p.tile_group) {
      int tm, tn;
      tile_coords(t, p, tm, tn);
      if (tile_group_of(p, tm) < 0) continue;
    }
    const int acc = it % C::ACC_STAGES;
    const uint32_t acc_phase = (it / C::ACC_STAGES) & 1;
    ++it;
    if (!mbar_wait(&sh.tempty[acc], acc_phase ^ 1, &sh.abort_flag, &g_err, 3)) return;
    tc_fence_after();
    const uint32_t d_tmem = sh.tmem_base + acc * C::ACC_COLS;
    for (int kb = 0; kb < p.num_k; ++kb) {
      if (!mbar_wait(&sh.full[stage], phase, &sh.abort_flag, &g_err, 4)) return;
      tc_fence_after();
      const uint32_t a_addr = smem_u32(sA + stage * A_BYTES);
      const uint32_t b_addr = smem_u32(sB + stage * C::B_BYTES);
      const uint32_t sf_addr = smem_u32(sSF + stage * C::SF_STAGE);
      const uint32_t tsfa = sh.tmem_base + C::SF_COL0 + stage * C::SF_COLS_PER_STAGE;
      const uint32_t tsfb = tsfa + 4;
      // scale records -> TMEM; tcgen05 operations of this thread execute in issue order,
      // so the copies land before the MMAs below read them
      tmem_cp_32x128b_x4(tsfa, sf_desc(sf_addr));
#pragma unroll
      for (int r = 0; r < BN / 128; ++r) tmem_cp_32x128b_x4(tsfb + 4 * r, sf_desc(sf_addr + (1 + r) * SF_BYTES));
#pragma unroll
      for (int j = 0; j < BK / 32; ++j) {
        const uint64_t ad = umma_desc_sw128(a_addr + j * 32, 16, 1024);
        const uint64_t bd = umma_desc_sw128(b_addr + j * 32, 16, 1024);
        umma_mx(d_tmem, ad, bd, idesc_mx(BM, BN, j, j), tsfa, tsfb, (kb | j) != 0 ? 1u : 0u);
      }
      umma_commit(&sh.empty[stage]);
      if (++stage == C::STAGES) {
        stage = 0;
        phase ^= 1;
      }
    }
    umma_commit(&sh.tfull[acc]);
  }
}

// 32 accumulator columns of one output row -> bf16, times the optional row / column scales
__device__ __forceinline__ void store_row32(__nv_bfloat16* drow, int col, const Params& p, bool vec_ok, float fr,
                                            const uint32_t* r) {
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) * fr;
  if (p.sb) {
    if (p.sb_rows) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] *= (col + j < p.N) ? __ldg(p.sb + col + j) : 0.f;
    } else {
      const float s = __ldg(p.sb);
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] *= s;
    }
  }
  if (vec_ok && col + 32 <= p.N) {
    uint4* dst = reinterpret_cast<uint4*>(drow + col);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 o;
      o.x = pack_bf16x2(v[8 * q + 0], v[8 * q + 1]);
      o.y = pack_bf16x2(v[8 * q + 2], v[8 * q + 3]);
      o.z = pack_bf16x2(v[8 * q + 4], v[8 * q + 5]);
      o.w = pack_bf16x2(v[8 * q + 6], v[8 * q + 7]);
      dst[q] = o;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (col + j < p.N) drow[col + j] = __float2bfloat16(v[j]);
  }
}

template <int BN>
__device__ __forceinline__ void run_epilogue(const Params& p, Shared& sh, int warp, int lane) {
  using C = Cfg<BN>;
  const int q = warp & 3;                                   // TMEM lane quarter this warp may access
  constexpr int COLS = BN / (C::EPI_WARPS / 4);             // accumulator columns of this warp
  const int col0 = ((warp - 2) / 4) * COLS;
  int it = 0;
  const int tiles = p.num_m * p.num_n;
  const bool vec_ok = (p.ldd % 8) == 0;
  for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
    int tm, tn;
    tile_coords(t, p, tm, tn);
    if (tile_group_of(p, tm) < 0) continue;
    const int row = tm * BM + q * 32 + lane;
    __nv_bfloat16* drow = p.D + static_cast<size_t>(row) * p.ldd;
    const int acc = it % C::ACC_STAGES;
    const uint32_t acc_phase = (it / C::ACC_STAGES) & 1;
    ++it;
    if (!mbar_wait(&sh.tfull[acc], acc_phase, &sh.abort_flag, &g_err, 5)) return;
    tc_fence_after();
    const float fr = !p.sa ? 1.f : (p.sa_rows ? (row < p.M ? __ldg(p.sa + row) : 0.f) : __ldg(p.sa));
    const uint32_t tbase = sh.tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * C::ACC_COLS + col0;
    if constexpr (C::ACC_STAGES == 1) {
      // the whole slice into registers, release the accumulator, then convert and store
      uint32_t r[COLS];
#pragma unroll
      for (int c = 0; c < COLS / 32; ++c) tmem_ld_32x32b_x32(tbase + c * 32, *reinterpret_cast<uint32_t(*)[32]>(r + 32 * c));
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh.tempty[acc]);
      if (row < p.M) {
#pragma unroll
        for (int c = 0; c < COLS / 32; ++c) {
          const int col = tn * BN + col0 + c * 32;
          if (col < p.N) store_row32(drow, col, p, vec_ok, fr, r + 32 * c);
        }
      }
    } else {
#pragma unroll 1
      for (int c = 0; c < COLS / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tbase + c * 32, r);
        tmem_ld_wait();
        const int col = tn * BN + col0 + c * 32;
        if (row < p.M && col < p.N) store_row32(drow, col, p, vec_ok, fr, r);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh.tempty[acc]);
    }
  }
}

template <int BN>
__global__ void __launch_bounds__(Cfg<BN>::NUM_THREADS, 1)
    mx_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, Params p) {
  using C = Cfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ Shared sh;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::STAGES * A_BYTES;
  uint8_t* sSF = sB + C::STAGES * C::B_BYTES;  // 1024-aligned: the stage tiles are multiples of 16 KB
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&sh.full[s], 1);
      mbar_init(&sh.empty[s], 1);
    }
    for (int a = 0; a < C::ACC_STAGES; ++a) {
      mbar_init(&sh.tfull[a], 1);
      mbar_init(&sh.tempty[a], C::EPI_WARPS);
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
    if (lane == 0) run_producer<BN>(&tmA, &tmB, p, sh, sA, sB, sSF);
  } else if (warp == 1) {
    if (lane == 0) run_mma<BN>(p, sh, sA, sB, sSF);
  } else {
    run_epilogue<BN>(p, sh, warp, lane);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(sh.tmem_base, TMEM_COLS);
  }
}

template <int BN>
void launch_mx(const void* A, const void* B, const void* sfa, const void* sfb, void* D, int64_t M, int64_t N,
               int64_t K, cudaStream_t stream, const MxEpilogue& ep) {
  using C = Cfg<BN>;
  const CUtensorMap ta = make_tmap_u8_2d(A, M, K, K, BM, BK);
  const CUtensorMap tb = make_tmap_u8_2d(B, N * ep.num_groups, K, K, BN, BK);
  Params p;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.b_records = (int)((N + 127) / 128);
  p.num_m = (int)((M + BM - 1) / BM);
  p.num_n = (int)((N + BN - 1) / BN);
  p.num_k = (int)(K / BK);
  p.sfa = static_cast<const uint8_t*>(sfa);
  p.sfb = static_cast<const uint8_t*>(sfb);
  p.D = static_cast<__nv_bfloat16*>(D);
  p.ldd = (int)N;
  p.sf_unit = sfa == nullptr;
  if (p.sf_unit) {
    static bool unit_set = false;  // fill the unit record once per process
    if (!unit_set) {
      uint8_t host[SF_BYTES];
      for (int i = 0; i < SF_BYTES; ++i) host[i] = 127;
      check_cuda(cudaMemcpyToSymbol(g_unit_sf, host, SF_BYTES), "mx unit scales");
      unit_set = true;
    }
    void* unit = nullptr;
    check_cuda(cudaGetSymbolAddress(&unit, g_unit_sf), "mx unit scales address");
    p.sfa = p.sfb = static_cast<const uint8_t*>(unit);
  }
  p.sa = ep.sa;
  p.sb = ep.sb;
  p.sa_rows = ep.sa_rows;
  p.sb_rows = ep.sb_rows;
  p.tile_group = ep.tile_group;
  static bool attr_set = false;
  if (!attr_set) {
    check_cuda(cudaFuncSetAttribute(mx_gemm_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES),
               "mx gemm smem attr");
    attr_set = true;
  }
  static int sms = 0;
  if (sms == 0) {
    int dev;
    check_cuda(cudaGetDevice(&dev), "mx gemm dev");
    sms = num_sms(dev);
  }
  const int tiles = p.num_m * p.num_n;
  mx_gemm_kernel<BN><<<tiles < sms ? tiles : sms, C::NUM_THREADS, C::SMEM_BYTES, stream>>>(ta, tb, p);
  check_cuda(cudaGetLastError(), "mx gemm launch");
}

}  // namespace mx_impl

void gemm_mxfp8(const void* A, const void* B, const void* sfa, const void* sfb, void* D, int64_t M, int64_t N,
                int64_t K, cudaStream_t stream, int tile_n, const MxEpilogue& ep) {
  using namespace mx_impl;
  if (M == 0 || N == 0) return;
  if (K % BK) throw std::runtime_error("gemm_mxfp8: K must be a multiple of 128");
  if (M >= (1ll << 31) || N >= (1ll << 31) || K >= (1ll << 31)) throw std::runtime_error("gemm_mxfp8: dims");
  if ((sfa == nullptr) != (sfb == nullptr)) throw std::runtime_error("gemm_mxfp8: both or neither scale records");
  if ((reinterpret_cast<uintptr_t>(sfa) & 15) || (reinterpret_cast<uintptr_t>(sfb) & 15))
    throw std::runtime_error("gemm_mxfp8: scale records must be 16-byte aligned");
  if (ep.tile_group != nullptr && (N % 128 || ep.num_groups < 1))
    throw std::runtime_error("gemm_mxfp8 grouped: N per group must be a multiple of 128");
  if (tile_n == 0) tile_n = N >= 256 ? 256 : 128;  // the wide tile wherever N has 256 columns
  if (tile_n == 256) launch_mx<256>(A, B, sfa, sfb, D, M, N, K, stream, ep);
  else if (tile_n == 128) launch_mx<128>(A, B, sfa, sfb, D, M, N, K, stream, ep);
  else throw std::runtime_error("gemm_mxfp8: tile_n must be 0, 128 or 256");
}

int mxgemm_error_code(bool reset) {
  int v = 0;
  check_cuda(cudaMemcpyFromSymbol(&v, mx_impl::g_err, sizeof(int)), "mx gemm error read");
  if (reset) {
    int z = 0;
    check_cuda(cudaMemcpyToSymbol(mx_impl::g_err, &z, sizeof(int)), "mx gemm error reset");
  }
  return v;
}

}  // namespace ttb
