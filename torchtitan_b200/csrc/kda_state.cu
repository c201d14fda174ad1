// Inter-chunk state recurrence of chunked KDA (Kimi Delta Attention) on tcgen05.
//
// Per head, chunks n = 0..NT-1 of C = 64 tokens, state S_n in R^{K x V} (K = V = 128):
//   forward   v'_n    = u_n - w_n S_n
//             S_{n+1} = diag(d_n) S_n + kdec_n^T v'_n
//   backward  dv'_n   = Aqk_n^T dO_n + kdec_n dS_{n+1}
//             dS_n    = diag(d_n) dS_{n+1} + qg_n^T dO_n - w_n^T dv'_n
// Only these recurrences are sequential.  The kernels emit the per-chunk states (S_n, and
// dS_{n+1} in the backward) and v' / dv'; everything else (o = qg S + Aqk v', and the
// gradients of qg, w, kdec, Aqk, d) is a batched GEMM over all chunks at once, done by the
// caller.  This is the state-passing split of the chunked delta rule (Yang et al. 2024).
//
// One CTA per head; the transposed state S^T [V x K] lives in TMEM as the fp32 accumulator
// (TMEM lane = v).  Per chunk:
//   compute warps: S^T -> registers -> bf16 operand tile in shared memory (and the chunk's
//                  state to global), then scale the TMEM copy by d_n;
//   MMA thread:    D1 = S^T w^T (+ for the backward dO^T Aqk) -> v'^T; then
//                  S^T += v'^T kdec  (backward: dS^T += dO^T qg - dv'^T w);
//   producer warp: TMA of the chunk's w / kdec / u^T (backward: qg, w, kdec, dO, Aqk) into a
//                  two-stage ring.
// bf16 operands with fp32 accumulation (the state itself stays fp32 in TMEM).  Every wait is
// bounded (sm100_ptx.cuh); on expiry the kernel records a code readable by
// kda_state_error_code() and unwinds, releasing TMEM.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <stdexcept>

#include "launch_api.h"
#include "sm100_ptx.cuh"
#include "tma_host.h"

namespace ttb {
namespace kstate {

__device__ int g_err;

constexpr int C = 64, K = 128, V = 128;
constexpr int NTHREADS = 192;  // warp 0 producer, warp 1 MMA + TMEM, warps 2..5 compute (lane = v)
constexpr int TILE_CK = C * K * 2;     // [C x K] bf16, two 64-column swizzled boxes
constexpr int TILE_VC = V * C * 2;     // [V x C] bf16, one 64-column swizzled box
constexpr int TILE_CV = C * V * 2;     // [C x V] bf16, two boxes
constexpr int TILE_CC = C * C * 2;     // [C x C] bf16, one box
constexpr int TILE_VK = V * K * 2;     // [V x K] bf16, two boxes

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ uint64_t desc_add(uint64_t d, uint32_t bytes) { return d + (bytes >> 4); }

__device__ __forceinline__ void tmem_st_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// row r, 16-byte unit j (8 bf16) of a [rows x 64] bf16 tile in the 128-byte-swizzled K-major layout
__device__ __forceinline__ uint4* sw128(uint8_t* tile, int r, int j) {
  return reinterpret_cast<uint4*>(tile + r * 128 + ((j ^ (r & 7)) << 4));
}

struct Bars {
  uint64_t full[2], empty[2];
  uint64_t sb_full, d1_full, vb_full, s_ready;
  uint32_t tmem_base;
  int abort_flag;
};

// the thread's 128-float state row: TMEM -> registers, in 32-column pieces
__device__ __forceinline__ void load_row(uint32_t taddr, float (&x)[K]) {
#pragma unroll
  for (int c = 0; c < K / 32; ++c) tmem_ld_32x32b_x32(taddr + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&x[c * 32]));
  tmem_ld_wait();
}

// state row -> global bf16 row, bf16 swizzled operand row (two 64-column boxes), then scale by d
// and write back to TMEM
__device__ __forceinline__ void stage_state_row(float (&x)[K], uint32_t taddr, uint8_t* sb, int r,
                                                __nv_bfloat16* grow, const float* d) {
#pragma unroll
  for (int j = 0; j < K / 8; ++j) {
    uint4 u;
    u.x = pack_bf16x2(x[8 * j], x[8 * j + 1]);
    u.y = pack_bf16x2(x[8 * j + 2], x[8 * j + 3]);
    u.z = pack_bf16x2(x[8 * j + 4], x[8 * j + 5]);
    u.w = pack_bf16x2(x[8 * j + 6], x[8 * j + 7]);
    *sw128(sb + (j >> 3) * (V * 128), r, j & 7) = u;
    reinterpret_cast<uint4*>(grow)[j] = u;
  }
#pragma unroll
  for (int c = 0; c < K / 32; ++c) {
    uint32_t o[32];
#pragma unroll
    for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(x[c * 32 + e] * __ldg(d + c * 32 + e));
    tmem_st_x32(taddr + c * 32, o);
  }
  tmem_st_wait();
}

struct FwdArgs {
  int BH, NT;
  const float* dec;     // [BH*NT, K]
  const float* S0;      // [BH, V, K] initial state (transposed), or null
  __nv_bfloat16* states;  // [BH*NT, V, K]  S_n^T at the start of chunk n
  __nv_bfloat16* vnT;     // [BH*NT, V, C]  v'_n^T
  float* Sfin;            // [BH, V, K]     final state (transposed), or null
};

__global__ void __launch_bounds__(NTHREADS, 1)
    state_fwd_kernel(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap tkd,
                     const __grid_constant__ CUtensorMap tuT, FwdArgs a) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ Bars bar;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int STAGE = 2 * TILE_CK + TILE_VC;  // w, kdec, u^T
  uint8_t* s_b = smem + 2 * STAGE;              // S^T operand [V x K]
  uint8_t* v_b = s_b + TILE_VK;                 // v'^T operand [V x C]
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int bh = blockIdx.x;
  const int NT = a.NT;
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar.full[i], 1);
      mbar_init(&bar.empty[i], 1);
    }
    mbar_init(&bar.sb_full, 4);
    mbar_init(&bar.d1_full, 1);
    mbar_init(&bar.vb_full, 4);
    mbar_init(&bar.s_ready, 1);
    bar.abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tw);
    tma_prefetch_desc(&tkd);
    tma_prefetch_desc(&tuT);
  }
  if (warp == 1) tmem_alloc(&bar.tmem_base, 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar.tmem_base;  // cols [0,128): S^T; [128,192): D1 = S^T w^T

  if (warp == 0) {
    if (lane == 0) {
      for (int n = 0; n < NT; ++n) {
        const int st = n & 1;
        if (!mbar_wait(&bar.empty[st], ((n >> 1) & 1) ^ 1, &bar.abort_flag, &g_err, 201)) break;
        uint8_t* s = smem + st * STAGE;
        const int row_ck = (bh * NT + n) * C, row_v = (bh * NT + n) * V;
        mbar_arrive_expect_tx(&bar.full[st], STAGE);
        tma_load_2d(s, &tw, &bar.full[st], 0, row_ck);
        tma_load_2d(s + C * 128, &tw, &bar.full[st], 64, row_ck);
        tma_load_2d(s + TILE_CK, &tkd, &bar.full[st], 0, row_ck);
        tma_load_2d(s + TILE_CK + C * 128, &tkd, &bar.full[st], 64, row_ck);
        tma_load_2d(s + 2 * TILE_CK, &tuT, &bar.full[st], 0, row_v);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_d1 = umma_idesc_bf16(V, C, false, false);  // [V x C] = S^T [V x K] . w^T
      constexpr uint32_t idesc_s = umma_idesc_bf16(V, K, false, true);    // [V x K] += v'^T [V x C] . kdec
      const uint32_t sb_addr = smem_u32(s_b), vb_addr = smem_u32(v_b);
      for (int n = 0; n < NT; ++n) {
        const int st = n & 1;
        const uint32_t w_addr = smem_u32(smem + st * STAGE), kd_addr = w_addr + TILE_CK;
        if (!mbar_wait(&bar.full[st], (n >> 1) & 1, &bar.abort_flag, &g_err, 202)) break;
        if (!mbar_wait(&bar.sb_full, n & 1, &bar.abort_flag, &g_err, 203)) break;
        tc_fence_after();
        const uint64_t da = umma_desc_sw128(sb_addr, 16, 1024), db = umma_desc_sw128(w_addr, 16, 1024);
#pragma unroll
        for (int kk = 0; kk < K / 16; ++kk)
          umma_bf16(tmem + 128, desc_add(da, (kk >> 2) * (V * 128) + (kk & 3) * 32),
                    desc_add(db, (kk >> 2) * (C * 128) + (kk & 3) * 32), idesc_d1, kk > 0 ? 1u : 0u);
        umma_commit(&bar.d1_full);
        if (!mbar_wait(&bar.vb_full, n & 1, &bar.abort_flag, &g_err, 204)) break;
        tc_fence_after();
        const uint64_t va = umma_desc_sw128(vb_addr, 16, 1024), kb = umma_desc_sw128(kd_addr, C * 128, 1024);
#pragma unroll
        for (int kk = 0; kk < C / 16; ++kk)
          umma_bf16(tmem, desc_add(va, kk * 32), desc_add(kb, kk * 2048), idesc_s, 1u);
        umma_commit(&bar.s_ready);
        umma_commit(&bar.empty[st]);
      }
    }
  } else {
    const int q = warp & 3;
    const int r = q * 32 + lane;  // v
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    const uint32_t s_col = tmem + lane_base, d1_col = tmem + lane_base + 128;
    float x[K];
    // initial state
    {
      if (a.S0 != nullptr) {
        const float4* src = reinterpret_cast<const float4*>(a.S0 + (static_cast<size_t>(bh) * V + r) * K);
#pragma unroll
        for (int j = 0; j < K / 4; ++j) {
          const float4 t = src[j];
          x[4 * j] = t.x, x[4 * j + 1] = t.y, x[4 * j + 2] = t.z, x[4 * j + 3] = t.w;
        }
      } else {
#pragma unroll
        for (int j = 0; j < K; ++j) x[j] = 0.f;
      }
    }
    bool ok = true;
    for (int n = 0; n < NT; ++n) {
      const int st = n & 1;
      const size_t bn = static_cast<size_t>(bh) * NT + n;
      if (n > 0) {
        if (!mbar_wait(&bar.s_ready, (n - 1) & 1, &bar.abort_flag, &g_err, 205)) { ok = false; break; }
        tc_fence_after();
        load_row(s_col, x);
      }
      stage_state_row(x, s_col, s_b, r, a.states + (bn * V + r) * K, a.dec + bn * K);
      fence_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar.sb_full);
      if (!mbar_wait(&bar.d1_full, n & 1, &bar.abort_flag, &g_err, 206)) { ok = false; break; }
      if (!mbar_wait(&bar.full[st], (n >> 1) & 1, &bar.abort_flag, &g_err, 207)) { ok = false; break; }
      tc_fence_after();
      uint32_t dd[64];
      tmem_ld_32x32b_x32(d1_col, *reinterpret_cast<uint32_t(*)[32]>(&dd[0]));
      tmem_ld_32x32b_x32(d1_col + 32, *reinterpret_cast<uint32_t(*)[32]>(&dd[32]));
      tmem_ld_wait();
      uint8_t* ut = smem + st * STAGE + 2 * TILE_CK;
      uint4* vrow = reinterpret_cast<uint4*>(a.vnT + (bn * V + r) * C);
#pragma unroll
      for (int j = 0; j < C / 8; ++j) {
        const uint4 uu = *sw128(ut, r, j);
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&uu);
        uint32_t pk[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(h[e]);
          pk[e] = pack_bf16x2(f.x - __uint_as_float(dd[8 * j + 2 * e]), f.y - __uint_as_float(dd[8 * j + 2 * e + 1]));
        }
        const uint4 o = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        *sw128(v_b, r, j) = o;
        vrow[j] = o;
      }
      fence_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar.vb_full);
    }
    if (ok && NT > 0 && a.Sfin != nullptr) {
      if (mbar_wait(&bar.s_ready, (NT - 1) & 1, &bar.abort_flag, &g_err, 208)) {
        tc_fence_after();
        load_row(s_col, x);
        float4* dst = reinterpret_cast<float4*>(a.Sfin + (static_cast<size_t>(bh) * V + r) * K);
#pragma unroll
        for (int j = 0; j < K / 4; ++j) dst[j] = make_float4(x[4 * j], x[4 * j + 1], x[4 * j + 2], x[4 * j + 3]);
      }
    } else if (NT == 0 && a.Sfin != nullptr) {
      float4* dst = reinterpret_cast<float4*>(a.Sfin + (static_cast<size_t>(bh) * V + r) * K);
#pragma unroll
      for (int j = 0; j < K / 4; ++j) dst[j] = make_float4(x[4 * j], x[4 * j + 1], x[4 * j + 2], x[4 * j + 3]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

struct BwdArgs {
  int BH, NT;
  const float* dec;       // [BH*NT, K]
  const float* dSfin;     // [BH, V, K] gradient of the final state (transposed), or null
  __nv_bfloat16* dstates;  // [BH*NT, V, K]  dS_{n+1}^T: the gradient entering chunk n from later chunks
  float* duT;              // [BH*NT, V, C]  dv'_n^T
  float* dS0;              // [BH, V, K]     gradient of the initial state (transposed), or null
};

__global__ void __launch_bounds__(NTHREADS, 1)
    state_bwd_kernel(const __grid_constant__ CUtensorMap tqg, const __grid_constant__ CUtensorMap tw,
                     const __grid_constant__ CUtensorMap tkd, const __grid_constant__ CUtensorMap tdo,
                     const __grid_constant__ CUtensorMap taqk, BwdArgs a) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ Bars bar;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int STAGE = 3 * TILE_CK + TILE_CV + TILE_CC;  // qg, w, kdec, dO, Aqk
  uint8_t* s_b = smem + 2 * STAGE;  // dS^T operand [V x K]
  uint8_t* v_b = s_b + TILE_VK;     // -dv'^T operand [V x C]
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int bh = blockIdx.x;
  const int NT = a.NT;
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar.full[i], 1);
      mbar_init(&bar.empty[i], 1);
    }
    mbar_init(&bar.sb_full, 4);
    mbar_init(&bar.d1_full, 1);
    mbar_init(&bar.vb_full, 4);
    mbar_init(&bar.s_ready, 1);
    bar.abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tqg);
    tma_prefetch_desc(&tw);
    tma_prefetch_desc(&tkd);
    tma_prefetch_desc(&tdo);
    tma_prefetch_desc(&taqk);
  }
  if (warp == 1) tmem_alloc(&bar.tmem_base, 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar.tmem_base;  // cols [0,128): dS^T; [128,192): D1 = dv'^T

  if (warp == 0) {
    if (lane == 0) {
      for (int i = 0; i < NT; ++i) {
        const int n = NT - 1 - i, st = i & 1;
        if (!mbar_wait(&bar.empty[st], ((i >> 1) & 1) ^ 1, &bar.abort_flag, &g_err, 211)) break;
        uint8_t* s = smem + st * STAGE;
        const int row_c = (bh * NT + n) * C;
        mbar_arrive_expect_tx(&bar.full[st], STAGE);
        tma_load_2d(s, &tqg, &bar.full[st], 0, row_c);
        tma_load_2d(s + C * 128, &tqg, &bar.full[st], 64, row_c);
        tma_load_2d(s + TILE_CK, &tw, &bar.full[st], 0, row_c);
        tma_load_2d(s + TILE_CK + C * 128, &tw, &bar.full[st], 64, row_c);
        tma_load_2d(s + 2 * TILE_CK, &tkd, &bar.full[st], 0, row_c);
        tma_load_2d(s + 2 * TILE_CK + C * 128, &tkd, &bar.full[st], 64, row_c);
        tma_load_2d(s + 3 * TILE_CK, &tdo, &bar.full[st], 0, row_c);
        tma_load_2d(s + 3 * TILE_CK + C * 128, &tdo, &bar.full[st], 64, row_c);
        tma_load_2d(s + 3 * TILE_CK + TILE_CV, &taqk, &bar.full[st], 0, row_c);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_dv_a = umma_idesc_bf16(V, C, true, true);    // dO^T [V x C] . Aqk
      constexpr uint32_t idesc_dv_b = umma_idesc_bf16(V, C, false, false);  // dS^T [V x K] . kdec^T
      constexpr uint32_t idesc_s = umma_idesc_bf16(V, K, true, true);       // dO^T [V x C] . qg
      constexpr uint32_t idesc_s2 = umma_idesc_bf16(V, K, false, true);     // (-dv'^T) [V x C] . w
      const uint32_t sb_addr = smem_u32(s_b), vb_addr = smem_u32(v_b);
      for (int i = 0; i < NT; ++i) {
        const int st = i & 1;
        const uint32_t qg_addr = smem_u32(smem + st * STAGE), w_addr = qg_addr + TILE_CK,
                       kd_addr = qg_addr + 2 * TILE_CK, do_addr = qg_addr + 3 * TILE_CK,
                       aq_addr = do_addr + TILE_CV;
        if (!mbar_wait(&bar.full[st], (i >> 1) & 1, &bar.abort_flag, &g_err, 212)) break;
        if (!mbar_wait(&bar.sb_full, i & 1, &bar.abort_flag, &g_err, 213)) break;
        tc_fence_after();
        // D1 = dO^T Aqk + dS^T kdec^T
        const uint64_t doa = umma_desc_sw128(do_addr, C * 128, 1024);  // A = dO^T, M-major (v contiguous)
        const uint64_t aqb = umma_desc_sw128(aq_addr, C * 128, 1024);  // B = Aqk as [N=j x K=i], N-major
#pragma unroll
        for (int kk = 0; kk < C / 16; ++kk)
          umma_bf16(tmem + 128, desc_add(doa, kk * 2048), desc_add(aqb, kk * 2048), idesc_dv_a, kk > 0 ? 1u : 0u);
        const uint64_t sa = umma_desc_sw128(sb_addr, 16, 1024), kdb = umma_desc_sw128(kd_addr, 16, 1024);
#pragma unroll
        for (int kk = 0; kk < K / 16; ++kk)
          umma_bf16(tmem + 128, desc_add(sa, (kk >> 2) * (V * 128) + (kk & 3) * 32),
                    desc_add(kdb, (kk >> 2) * (C * 128) + (kk & 3) * 32), idesc_dv_b, 1u);
        umma_commit(&bar.d1_full);
        // dS^T (already scaled by d) += dO^T qg
        const uint64_t qgb = umma_desc_sw128(qg_addr, C * 128, 1024);
#pragma unroll
        for (int kk = 0; kk < C / 16; ++kk)
          umma_bf16(tmem, desc_add(doa, kk * 2048), desc_add(qgb, kk * 2048), idesc_s, 1u);
        if (!mbar_wait(&bar.vb_full, i & 1, &bar.abort_flag, &g_err, 214)) break;
        tc_fence_after();
        // dS^T += (-dv'^T) w
        const uint64_t va = umma_desc_sw128(vb_addr, 16, 1024), wb = umma_desc_sw128(w_addr, C * 128, 1024);
#pragma unroll
        for (int kk = 0; kk < C / 16; ++kk)
          umma_bf16(tmem, desc_add(va, kk * 32), desc_add(wb, kk * 2048), idesc_s2, 1u);
        umma_commit(&bar.s_ready);
        umma_commit(&bar.empty[st]);
      }
    }
  } else {
    const int q = warp & 3;
    const int r = q * 32 + lane;  // v
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    const uint32_t s_col = tmem + lane_base, d1_col = tmem + lane_base + 128;
    float x[K];
    if (a.dSfin != nullptr) {
      const float4* src = reinterpret_cast<const float4*>(a.dSfin + (static_cast<size_t>(bh) * V + r) * K);
#pragma unroll
      for (int j = 0; j < K / 4; ++j) {
        const float4 t = src[j];
        x[4 * j] = t.x, x[4 * j + 1] = t.y, x[4 * j + 2] = t.z, x[4 * j + 3] = t.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < K; ++j) x[j] = 0.f;
    }
    bool ok = true;
    for (int i = 0; i < NT; ++i) {
      const int n = NT - 1 - i;
      const size_t bn = static_cast<size_t>(bh) * NT + n;
      if (i > 0) {
        if (!mbar_wait(&bar.s_ready, (i - 1) & 1, &bar.abort_flag, &g_err, 215)) { ok = false; break; }
        tc_fence_after();
        load_row(s_col, x);
      }
      stage_state_row(x, s_col, s_b, r, a.dstates + (bn * V + r) * K, a.dec + bn * K);
      fence_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar.sb_full);
      if (!mbar_wait(&bar.d1_full, i & 1, &bar.abort_flag, &g_err, 216)) { ok = false; break; }
      tc_fence_after();
      uint32_t dd[64];
      tmem_ld_32x32b_x32(d1_col, *reinterpret_cast<uint32_t(*)[32]>(&dd[0]));
      tmem_ld_32x32b_x32(d1_col + 32, *reinterpret_cast<uint32_t(*)[32]>(&dd[32]));
      tmem_ld_wait();
      float4* durow = reinterpret_cast<float4*>(a.duT + (bn * V + r) * C);
#pragma unroll
      for (int j = 0; j < C / 8; ++j) {
        float f[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(dd[8 * j + e]);
        durow[2 * j] = make_float4(f[0], f[1], f[2], f[3]);
        durow[2 * j + 1] = make_float4(f[4], f[5], f[6], f[7]);
        *sw128(v_b, r, j) = make_uint4(pack_bf16x2(-f[0], -f[1]), pack_bf16x2(-f[2], -f[3]), pack_bf16x2(-f[4], -f[5]),
                                       pack_bf16x2(-f[6], -f[7]));
      }
      fence_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar.vb_full);
    }
    if (a.dS0 != nullptr) {
      bool have = ok;
      if (ok && NT > 0) {
        have = mbar_wait(&bar.s_ready, (NT - 1) & 1, &bar.abort_flag, &g_err, 217);
        if (have) {
          tc_fence_after();
          load_row(s_col, x);
        }
      }
      if (have) {
        float4* dst = reinterpret_cast<float4*>(a.dS0 + (static_cast<size_t>(bh) * V + r) * K);
#pragma unroll
        for (int j = 0; j < K / 4; ++j) dst[j] = make_float4(x[4 * j], x[4 * j + 1], x[4 * j + 2], x[4 * j + 3]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

constexpr int FWD_SMEM = 2 * (2 * TILE_CK + TILE_VC) + TILE_VK + TILE_VC + 1024;
constexpr int BWD_SMEM = 2 * (3 * TILE_CK + TILE_CV + TILE_CC) + TILE_VK + TILE_VC + 1024;
static_assert(BWD_SMEM <= 227 * 1024, "shared memory");

}  // namespace kstate

void kda_state_fwd(const void* w, const void* kd, const void* uT, const float* dec, const float* S0, void* states,
                   void* vnT, float* Sfin, int BH, int NT, cudaStream_t s) {
  using namespace kstate;
  if (BH == 0) return;
  static bool attr = false;
  if (!attr) {
    check_cuda(cudaFuncSetAttribute(state_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, FWD_SMEM),
               "kda state smem");
    attr = true;
  }
  const uint64_t rows_c = static_cast<uint64_t>(BH) * NT * C, rows_v = static_cast<uint64_t>(BH) * NT * V;
  const CUtensorMap tw = make_tmap_bf16_2d(w, rows_c, K, K, C, 64);
  const CUtensorMap tkd = make_tmap_bf16_2d(kd, rows_c, K, K, C, 64);
  const CUtensorMap tuT = make_tmap_bf16_2d(uT, rows_v, C, C, V, 64);
  FwdArgs a{BH, NT, dec, S0, static_cast<__nv_bfloat16*>(states), static_cast<__nv_bfloat16*>(vnT), Sfin};
  state_fwd_kernel<<<BH, NTHREADS, FWD_SMEM, s>>>(tw, tkd, tuT, a);
  check_cuda(cudaGetLastError(), "kda state fwd launch");
}

void kda_state_bwd(const void* qg, const void* w, const void* kd, const void* dO, const void* Aqk, const float* dec,
                   const float* dSfin, void* dstates, float* duT, float* dS0, int BH, int NT, cudaStream_t s) {
  using namespace kstate;
  if (BH == 0) return;
  static bool attr = false;
  if (!attr) {
    check_cuda(cudaFuncSetAttribute(state_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, BWD_SMEM),
               "kda state bwd smem");
    attr = true;
  }
  const uint64_t rows_c = static_cast<uint64_t>(BH) * NT * C;
  const CUtensorMap tqg = make_tmap_bf16_2d(qg, rows_c, K, K, C, 64);
  const CUtensorMap tw = make_tmap_bf16_2d(w, rows_c, K, K, C, 64);
  const CUtensorMap tkd = make_tmap_bf16_2d(kd, rows_c, K, K, C, 64);
  const CUtensorMap tdo = make_tmap_bf16_2d(dO, rows_c, V, V, C, 64);
  const CUtensorMap taqk = make_tmap_bf16_2d(Aqk, rows_c, C, C, C, 64);
  BwdArgs a{BH, NT, dec, dSfin, static_cast<__nv_bfloat16*>(dstates), duT, dS0};
  state_bwd_kernel<<<BH, NTHREADS, BWD_SMEM, s>>>(tqg, tw, tkd, tdo, taqk, a);
  check_cuda(cudaGetLastError(), "kda state bwd launch");
}

int kda_state_error_code(bool reset) {
  int v = 0;
  check_cuda(cudaMemcpyFromSymbol(&v, kstate::g_err, sizeof(int)), "kda state error read");
  if (reset && v) {
    int z = 0;
    check_cuda(cudaMemcpyToSymbol(kstate::g_err, &z, sizeof(int)), "kda state error reset");
  }
  return v;
}

}  // namespace ttb
