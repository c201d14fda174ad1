// Tensor-parallel GEMMs fused with their collectives over NVLink peer memory (sm_100a).
//
//   ag_gemm : D[tp*Ms, N] = AllGather_rows(X_r[Ms, K]) . B      (column-parallel linear with a
//             sequence-sharded input; B = W [N, K] or [K, N])
//   gemm_rs : out_r[Ms, N] = ReduceScatter_rows(X[tp*Ms, K] . B)  (row-parallel linear with a
//             sequence-sharded output)
//
// One persistent tcgen05 GEMM per call (tile 128 x 256 x 64, 4-stage TMA ring, accumulators in
// TMEM, one CTA per SM, all CTAs co-resident through a cooperative launch), with the collective
// done by the same kernel:
//
// ag_gemm: two copy warps per CTA pull their slice of every peer's shard over NVLink (16-byte
//   P2P loads) into a local landing buffer [tp*Ms, K], chunk by chunk starting with the next
//   rank, and count finished slices per chunk. The TMA producer works on this rank's own rows
//   first (straight from its shard) and waits, bounded, for a chunk's counter before loading
//   that chunk's rows from the landing buffer; so the transfer of chunk c+1 overlaps the MMAs of
//   chunk c and no TMA load ever reads another GPU's memory. The landing buffer doubles as the
//   gathered input the weight gradient needs.
// gemm_rs: tiles whose rows belong to other ranks run first; their epilogue stores the bf16
//   partial tile straight into the owner's receive slot (P2P stores), double-buffered by call
//   parity. Every CTA then adds one to every rank's completion counter (system-scope reduction);
//   once a rank's counter reaches tp x grid, its CTAs sum the tp partials of their slice of its
//   rows into the output.
//
// Cross-rank order: each rank signals "entered call e" (its shard is ready) and, for ag_gemm,
// "finished reading every peer in call e"; a rank leaves the kernel only when every peer is done
// with its shard, so the caller may overwrite the shard after the kernel. All waits are bounded
// (they record a code readable through tp_gemm_error_code() and let the kernel finish early).
// Plain P2P loads and stores only: no multicast, no NVLS.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <stdexcept>
#include <string>

#include "launch_api.h"
#include "sm100_ptx.cuh"
#include "tma_host.h"

namespace ttb {
namespace tpg {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;
constexpr int B_BYTES = BN * BK * 2;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024;
constexpr int NUM_THREADS = 256;  // w0 TMA, w1 MMA + TMEM, w2..5 epilogue, w6..7 copy / signalling
constexpr int GROUP_M = 8;
constexpr int MAX_TP = 8;
constexpr uint64_t kLimitNs = 20000000000ull;

__device__ int g_err;

struct Params {
  int mode;  // 0 ag_gemm, 1 gemm_rs
  int M, N, K, Ms;
  int num_m, num_n, num_k;
  int tp, rank;
  uint32_t epoch;
  // ag_gemm
  const __nv_bfloat16* shard[MAX_TP];  // every rank's input shard [Ms, K] (peer mappings)
  __nv_bfloat16* land;                 // local landing buffer [M, K]
  unsigned* chunk_ready;               // local [MAX_TP] counters (zeroed before the launch)
  __nv_bfloat16* D;                    // ag_gemm output [M, N]
  // gemm_rs
  __nv_bfloat16* recv[MAX_TP];  // every rank's receive area [2][tp][Ms, N] (peer mappings)
  unsigned* done[MAX_TP];       // every rank's completion counters [2] (peer mappings)
  __nv_bfloat16* out;           // gemm_rs output [Ms, N]
  int parity;
  // signalling: every rank's pad of 2*MAX_TP words: [0, tp) "entered", [MAX_TP, MAX_TP+tp) "read done"
  unsigned* sig[MAX_TP];
};

struct Shared {
  uint64_t full[STAGES], empty[STAGES], tfull[2], tempty[2];
  uint32_t tmem_base;
  int abort_flag;
};

__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void red_release_sys_add(unsigned* p, unsigned v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// bounded wait until *p >= target (signed compare of the difference); false on expiry
template <bool SYS>
__device__ bool wait_geq(const unsigned* p, unsigned target, int code, volatile int* abort) {
  const uint64_t t0 = now_ns();
  while (true) {
    const unsigned v = SYS ? ld_acquire_sys(p) : ld_acquire_gpu(p);
    if (static_cast<int>(v - target) >= 0) return true;
    if ((abort && *abort) || now_ns() - t0 > kLimitNs || *static_cast<volatile int*>(&g_err) != 0) {
      atomicCAS(&g_err, 0, code);
      if (abort) *abort = 1;
      return false;
    }
    __nanosleep(64);
  }
}

// Tile order: chunk-major. ag_gemm starts with this rank's rows (no wait), then the next ranks;
// gemm_rs starts with the next rank's rows and ends with its own (their partials stay local).
struct Tile {
  int tm, tn, chunk;
};
__device__ __forceinline__ Tile tile_of(int t, const Params& p) {
  const int mt_per_chunk = p.Ms / BM;
  const int per_chunk = mt_per_chunk * p.num_n;
  const int ci = t / per_chunk;
  const int chunk = p.mode == 0 ? (p.rank + ci) % p.tp : (p.rank + 1 + ci) % p.tp;
  const int r = t - ci * per_chunk;
  const int band = GROUP_M * p.num_n;
  const int g = r / band;
  const int first = g * GROUP_M;
  const int gs = min(mt_per_chunk - first, GROUP_M);
  const int rr = r - g * band;
  Tile tl;
  tl.tm = chunk * mt_per_chunk + first + rr % gs;
  tl.tn = rr / gs;
  tl.chunk = chunk;
  return tl;
}

template <bool B_MN>
__device__ void run_producer(const CUtensorMap* tmOwn, const CUtensorMap* tmLand, const CUtensorMap* tmB,
                             const Params& p, Shared& sh, uint8_t* sA, uint8_t* sB) {
  int stage = 0;
  uint32_t phase = 0;
  const int tiles = p.num_m * p.num_n;
  int ready_chunk = -1;
  for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
    const Tile tl = tile_of(t, p);
    const bool own = p.mode == 1 || tl.chunk == p.rank;
    if (p.mode == 0 && !own && tl.chunk != ready_chunk) {
      // every CTA's copy warps have landed their slice of this chunk
      if (!wait_geq<false>(p.chunk_ready + tl.chunk, gridDim.x, 301, &sh.abort_flag)) return;
      fence_proxy_async_global();  // generic-proxy stores of the landing buffer -> TMA reads
      ready_chunk = tl.chunk;
    }
    for (int kb = 0; kb < p.num_k; ++kb) {
      if (!mbar_wait(&sh.empty[stage], phase ^ 1, &sh.abort_flag, &g_err, 302)) return;
      mbar_arrive_expect_tx(&sh.full[stage], STAGE_BYTES);
      uint8_t* a = sA + stage * A_BYTES;
      uint8_t* b = sB + stage * B_BYTES;
      const int k0 = kb * BK;
      if (p.mode == 0 && own) tma_load_2d(a, tmOwn, &sh.full[stage], k0, tl.tm * BM - p.rank * p.Ms);
      else tma_load_2d(a, p.mode == 0 ? tmLand : tmOwn, &sh.full[stage], k0, tl.tm * BM);
      if constexpr (!B_MN) {
        tma_load_2d(b, tmB, &sh.full[stage], k0, tl.tn * BN);
      } else {
#pragma unroll
        for (int j = 0; j < BN / 64; ++j) tma_load_2d(b + j * 8192, tmB, &sh.full[stage], tl.tn * BN + j * 64, k0);
      }
      if (++stage == STAGES) {
        stage = 0;
        phase ^= 1;
      }
    }
  }
  for (int s = 0; s < STAGES; ++s) {  // drain
    if (!mbar_wait(&sh.empty[stage], phase ^ 1, &sh.abort_flag, &g_err, 303)) return;
    if (++stage == STAGES) {
      stage = 0;
      phase ^= 1;
    }
  }
}

template <bool B_MN>
__device__ void run_mma(const Params& p, Shared& sh, uint8_t* sA, uint8_t* sB) {
  constexpr uint32_t idesc = umma_idesc_bf16(BM, BN, false, B_MN);
  int stage = 0;
  uint32_t phase = 0;
  int it = 0;
  const int tiles = p.num_m * p.num_n;
  for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
    const int acc = it & 1;
    const uint32_t acc_phase = (it >> 1) & 1;
    ++it;
    if (!mbar_wait(&sh.tempty[acc], acc_phase ^ 1, &sh.abort_flag, &g_err, 304)) return;
    tc_fence_after();
    const uint32_t d_tmem = sh.tmem_base + acc * BN;
    for (int kb = 0; kb < p.num_k; ++kb) {
      if (!mbar_wait(&sh.full[stage], phase, &sh.abort_flag, &g_err, 305)) return;
      tc_fence_after();
      const uint64_t ad0 = umma_desc_sw128(smem_u32(sA + stage * A_BYTES), 16, 1024);
      const uint64_t bd0 = B_MN ? umma_desc_sw128(smem_u32(sB + stage * B_BYTES), 8192, 1024)
                                : umma_desc_sw128(smem_u32(sB + stage * B_BYTES), 16, 1024);
#pragma unroll
      for (int k = 0; k < BK / 16; ++k)
        umma_bf16(d_tmem, ad0 + static_cast<uint64_t>((k * 32) >> 4),
                  bd0 + static_cast<uint64_t>((B_MN ? k * 2048 : k * 32) >> 4), idesc, (kb | k) != 0 ? 1u : 0u);
      umma_commit(&sh.empty[stage]);
      if (++stage == STAGES) {
        stage = 0;
        phase ^= 1;
      }
    }
    umma_commit(&sh.tfull[acc]);
  }
}

__device__ void run_epilogue(const Params& p, Shared& sh, int warp, int lane) {
  const int q = warp & 3;
  int it = 0;
  const int tiles = p.num_m * p.num_n;
  for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
    const Tile tl = tile_of(t, p);
    const int row = tl.tm * BM + q * 32 + lane;
    __nv_bfloat16* drow;
    if (p.mode == 0) {
      drow = p.D + static_cast<size_t>(row) * p.N;
    } else {  // partial tile to the owner's receive slot [parity][this rank][row - chunk*Ms]
      const size_t slot = (static_cast<size_t>(p.parity) * p.tp + p.rank) * p.Ms;
      drow = p.recv[tl.chunk] + (slot + (row - tl.chunk * p.Ms)) * p.N;
    }
    const int acc = it & 1;
    const uint32_t acc_phase = (it >> 1) & 1;
    ++it;
    if (!mbar_wait(&sh.tfull[acc], acc_phase, &sh.abort_flag, &g_err, 306)) return;
    tc_fence_after();
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(sh.tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN + c * 32, r);
      tmem_ld_wait();
      const int col = tl.tn * BN + c * 32;
      if (col < p.N) {  // N is a multiple of 32 (host check)
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
      }
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&sh.tempty[acc]);
  }
}

// ag_gemm copy warps (64 threads): this CTA's row slice of every chunk, next ranks first
__device__ void run_copy(const Params& p, Shared& sh, int tid) {
  const int rows_per = (p.Ms + gridDim.x - 1) / gridDim.x;
  const int r0 = blockIdx.x * rows_per, r1 = min(p.Ms, r0 + rows_per);
  const int vecs = p.K / 8;  // 16-byte vectors per row
  for (int i = 1; i <= p.tp; ++i) {
    const int c = (p.rank + i) % p.tp;  // i == tp: own chunk (local copy, for the backward)
    if (c != p.rank && tid == 0 && !wait_geq<true>(p.sig[p.rank] + c, p.epoch, 311, &sh.abort_flag)) {
      // peer never entered this call: count the slice anyway so the producer does not wait
      // a second limit; the error code is already set
    }
    asm volatile("bar.sync 1, 64;" ::: "memory");
    const uint4* src = reinterpret_cast<const uint4*>(p.shard[c]);
    uint4* dst = reinterpret_cast<uint4*>(p.land + static_cast<size_t>(c) * p.Ms * p.K);
    if (*static_cast<volatile int*>(&g_err) == 0) {
      // 8 independent 16-byte loads in flight per thread: NVLink latency, not issue, would
      // otherwise bound the copy
      constexpr int U = 8;
      const int64_t n = static_cast<int64_t>(r1 - r0) * vecs, base = static_cast<int64_t>(r0) * vecs;
      int64_t x = tid;
      for (; x + (U - 1) * 64 < n; x += U * 64) {
        uint4 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u)
          asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];"
                       : "=r"(v[u].x), "=r"(v[u].y), "=r"(v[u].z), "=r"(v[u].w)
                       : "l"(src + base + x + u * 64));
#pragma unroll
        for (int u = 0; u < U; ++u) dst[base + x + u * 64] = v[u];
      }
      for (; x < n; x += 64) {
        uint4 v;
        asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                     : "l"(src + base + x));
        dst[base + x] = v;
      }
    }
    __threadfence();
    asm volatile("bar.sync 1, 64;" ::: "memory");
    if (tid == 0) atomicAdd(p.chunk_ready + c, 1u);
  }
}

template <bool B_MN>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    tp_gemm_kernel(const __grid_constant__ CUtensorMap tmOwn, const __grid_constant__ CUtensorMap tmLand,
                   const __grid_constant__ CUtensorMap tmB, Params p) {
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
    if (p.mode == 1 && blockIdx.x == 0) {
      // reset this rank's counter of the NEXT call (other parity). Its last use (the previous
      // call) is over, and no peer can add to it before finishing this call, which waits for
      // this rank's increments; those are issued after this CTA's __syncthreads below.
      p.done[p.rank][p.parity ^ 1] = 0u;
    }
  }
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    // this rank's shard (ag) / receive slots (rs) are ready for the call: tell every peer
    __threadfence_system();
    for (int j = 0; j < p.tp; ++j) st_release_sys(p.sig[j] + p.rank, p.epoch);
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmOwn);
    tma_prefetch_desc(&tmB);
    if (p.mode == 0) tma_prefetch_desc(&tmLand);
  }
  if (warp == 1) tmem_alloc(&sh.tmem_base, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  if (warp == 0) {
    if (lane == 0) run_producer<B_MN>(&tmOwn, &tmLand, &tmB, p, sh, sA, sB);
  } else if (warp == 1) {
    if (lane == 0) run_mma<B_MN>(p, sh, sA, sB);
  } else if (warp < 6) {
    run_epilogue(p, sh, warp, lane);
    if (p.mode == 1) {
      // partials of this CTA are out: count it at every rank, then reduce this rank's rows
      asm volatile("bar.sync 2, 128;" ::: "memory");
      const int tid = threadIdx.x - 64;
      if (tid == 0) {
        __threadfence_system();
        for (int j = 0; j < p.tp; ++j) red_release_sys_add(p.done[j] + p.parity, 1u);
        wait_geq<true>(p.done[p.rank] + p.parity, static_cast<unsigned>(p.tp) * gridDim.x, 321, &sh.abort_flag);
      }
      asm volatile("bar.sync 2, 128;" ::: "memory");
      if (*static_cast<volatile int*>(&g_err) == 0) {
        const int rows_per = (p.Ms + gridDim.x - 1) / gridDim.x;
        const int r0 = blockIdx.x * rows_per, r1 = min(p.Ms, r0 + rows_per);
        const int vecs = p.N / 8;
        const __nv_bfloat16* base = p.recv[p.rank] + static_cast<size_t>(p.parity) * p.tp * p.Ms * p.N;
        for (int64_t x = tid; x < static_cast<int64_t>(r1 - r0) * vecs; x += 128) {
          const int64_t e = (static_cast<int64_t>(r0) * vecs + x) * 8;
          float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
          for (int s = 0; s < p.tp; ++s) {
            uint4 v;
            asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];"
                         : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                         : "l"(base + static_cast<size_t>(s) * p.Ms * p.N + e));
            const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const float2 f = __bfloat1622float2(h[u]);
              acc[2 * u] += f.x;
              acc[2 * u + 1] += f.y;
            }
          }
          uint4 o;
          o.x = pack_bf16x2(acc[0], acc[1]);
          o.y = pack_bf16x2(acc[2], acc[3]);
          o.z = pack_bf16x2(acc[4], acc[5]);
          o.w = pack_bf16x2(acc[6], acc[7]);
          *reinterpret_cast<uint4*>(p.out + e) = o;
        }
      }
    }
  } else if (p.mode == 0) {
    const int tid = threadIdx.x - 192;
    run_copy(p, sh, tid);
    if (blockIdx.x == 0) {
      // every chunk landed here: tell the peers this rank is done reading them, then wait until
      // every peer is done reading this rank's shard (after that the caller may overwrite it)
      if (tid == 0) {
        wait_geq<false>(p.chunk_ready + p.rank, gridDim.x, 312, nullptr);
        for (int c = 0; c < p.tp; ++c) wait_geq<false>(p.chunk_ready + c, gridDim.x, 313, nullptr);
        __threadfence_system();
        for (int j = 0; j < p.tp; ++j) st_release_sys(p.sig[j] + MAX_TP + p.rank, p.epoch);
        for (int j = 0; j < p.tp; ++j) wait_geq<true>(p.sig[p.rank] + MAX_TP + j, p.epoch, 314, nullptr);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(sh.tmem_base, 512);
  }
}

}  // namespace tpg

void tp_gemm(int mode, const void* const* shards, void* land, unsigned* chunk_ready, void* D, const void* B, bool b_mn,
             void* const* recv, unsigned* const* done, void* out, int parity, unsigned* const* sig, int tp, int rank,
             uint32_t epoch, int64_t Ms, int64_t N, int64_t K, cudaStream_t s) {
  using namespace tpg;
  if (tp < 1 || tp > MAX_TP || rank < 0 || rank >= tp) throw std::runtime_error("tp_gemm: tp must be 1..8");
  if (Ms % BM || N % 32 || K % 64 || N % 8)
    throw std::runtime_error("tp_gemm: rows per rank must be a multiple of 128, N of 32 and K of 64");
  Params p{};
  p.mode = mode;
  p.M = static_cast<int>(Ms * tp);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.Ms = static_cast<int>(Ms);
  p.num_m = p.M / BM;
  p.num_n = static_cast<int>((N + BN - 1) / BN);
  p.num_k = p.K / BK;
  p.tp = tp;
  p.rank = rank;
  p.epoch = epoch;
  for (int j = 0; j < tp; ++j) {
    p.sig[j] = sig[j];
    if (mode == 0) p.shard[j] = static_cast<const __nv_bfloat16*>(shards[j]);
    else {
      p.recv[j] = static_cast<__nv_bfloat16*>(recv[j]);
      p.done[j] = done[j];
    }
  }
  p.land = static_cast<__nv_bfloat16*>(land);
  p.chunk_ready = chunk_ready;
  p.D = static_cast<__nv_bfloat16*>(D);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.parity = parity;
  // A: ag -> this rank's shard (own rows) and the landing buffer; rs -> the local input [M, K]
  const CUtensorMap tmOwn = mode == 0 ? make_tmap_bf16_2d(shards[rank], Ms, K, K, BM, 64)
                                      : make_tmap_bf16_2d(shards[rank], Ms * tp, K, K, BM, 64);
  const CUtensorMap tmLand = mode == 0 ? make_tmap_bf16_2d(land, Ms * tp, K, K, BM, 64) : tmOwn;
  const CUtensorMap tmB = b_mn ? make_tmap_bf16_2d(B, K, N, N, 64, 64) : make_tmap_bf16_2d(B, N, K, K, BN, 64);
  static int sms = 0;
  if (sms == 0) {
    int dev;
    check_cuda(cudaGetDevice(&dev), "tp_gemm dev");
    sms = num_sms(dev);
  }
  const int tiles = p.num_m * p.num_n;
  // the same grid on every rank (same shapes), all CTAs resident at once
  const int grid = tiles < sms ? tiles : sms;
  void* args[] = {const_cast<CUtensorMap*>(&tmOwn), const_cast<CUtensorMap*>(&tmLand), const_cast<CUtensorMap*>(&tmB),
                  &p};
  if (b_mn) {
    static bool attr = false;
    if (!attr) {
      check_cuda(cudaFuncSetAttribute(tp_gemm_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES),
                 "tp_gemm smem");
      attr = true;
    }
    check_cuda(cudaLaunchCooperativeKernel(reinterpret_cast<void*>(tp_gemm_kernel<true>), grid, NUM_THREADS, args,
                                           SMEM_BYTES, s), "tp_gemm launch");
  } else {
    static bool attr = false;
    if (!attr) {
      check_cuda(cudaFuncSetAttribute(tp_gemm_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES),
                 "tp_gemm smem");
      attr = true;
    }
    check_cuda(cudaLaunchCooperativeKernel(reinterpret_cast<void*>(tp_gemm_kernel<false>), grid, NUM_THREADS, args,
                                           SMEM_BYTES, s), "tp_gemm launch");
  }
}

int tp_gemm_error_code(bool reset) {
  int v = 0;
  check_cuda(cudaMemcpyFromSymbol(&v, tpg::g_err, sizeof(int)), "tp_gemm error read");
  if (reset && v) {
    int z = 0;
    check_cuda(cudaMemcpyToSymbol(tpg::g_err, &z, sizeof(int)), "tp_gemm error reset");
  }
  return v;
}

}  // namespace ttb
