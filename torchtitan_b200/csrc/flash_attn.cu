// Flash attention for sm_100a on tcgen05 (forward) with GQA and a
// bottom-right-aligned causal mask (query i sees keys j <= i + Sk - Sq).
//
// Layout: q [B,Sq,H,Dqk], k [B,Sk,Hk,Dqk], v [B,Sk,Hk,Dv] bf16; o like q
// with Dv; lse [B,H,Sq] fp32 (natural log).
//
// Forward CTA = one 128-query tile of one head; warps:
//   0      TMA producer: Q once, then K/V tiles into a 2-stage ring
//   1      TMEM allocator + MMA issuer: S_j = Q K_j^T -> TMEM (2 buffers),
//          PV_j = P_j V_j -> TMEM (2 buffers)
//   2..5   softmax: thread r owns query row r; reads S_j from TMEM (two
//          passes: row max, then exp2 + row sum), writes P_j (bf16) into a
//          128B-swizzled smem tile (2 buffers) for the PV MMA, and folds
//          PV_{j-1} into its fp32 O row kept in registers.
// The MMA warp interleaves S_{j+1} and PV_{j-1} so the tensor cores work
// while the softmax warps process tile j.  All waits are bounded.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <stdexcept>

#include "launch_api.h"
#include "sm100_ptx.cuh"
#include "tma_host.h"

namespace ttb {
namespace attn_impl {

__device__ int g_err;


// lse / delta rows are padded to a multiple of 64 queries (zero-filled by the
// allocator) so 64-query slices can be bulk-copied without running off a row
__host__ __device__ __forceinline__ int lse_stride(int Sq) { return (Sq + 63) / 64 * 64; }

__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

constexpr int BM = 128;  // queries per CTA
constexpr int NUM_SM_WARPS = 8;                    // softmax / epilogue warps
constexpr int NUM_THREADS = 64 + 32 * NUM_SM_WARPS;  // + producer + MMA warp

template <int DQK, int DV, int BN>
struct Cfg {
  static constexpr int Q_BYTES = BM * DQK * 2;
  static constexpr int K_BYTES = BN * DQK * 2;
  static constexpr int V_BYTES = BN * DV * 2;
  static constexpr int P_BYTES = BM * BN * 2;
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = Q_OFF + Q_BYTES;
  static constexpr int V_OFF = K_OFF + 2 * K_BYTES;
  static constexpr int P_OFF = V_OFF + 2 * V_BYTES;
  static constexpr int RED_OFF = P_OFF + 2 * P_BYTES;      // float [2 stages][2 halves][BM] row maxima
  static constexpr int BAR_OFF = RED_OFF + 2 * 2 * BM * 4;  // struct Bars
  static constexpr int SMEM = BAR_OFF + 256;                // dynamic base is 1024-aligned (checked)
  static constexpr int S_COL = 0;        // 2 x BN columns
  static constexpr int PV_COL = 2 * BN;  // 2 x DV columns
  static constexpr int TMEM_COLS = 512;
  static_assert(2 * BN + 2 * DV <= 512, "TMEM budget");
  static_assert(DQK % 64 == 0 && DV % 64 == 0 && BN % 64 == 0, "tile dims");
};

struct Params {
  int B, Sq, Sk, H, Hk;
  int causal;
  float scale_log2;  // softmax scale * log2(e)
  __nv_bfloat16* o;
  float* lse;
  int num_qtiles;
  // packed documents (self-attention, optional): per token, the first position of its document
  // and one past its last; a query sees only keys of its own document
  const int* doc_start;
  const int* doc_end;
};

struct Bars {
  uint64_t q_full;
  uint64_t k_full[2], v_full[2], kv_empty[2];
  uint64_t s_full[2], s_free[2];
  uint64_t p_full[2], p_empty[2];
  uint64_t pv_full[2], pv_free[2];
  uint32_t tmem_base;
  int abort_flag;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void named_bar_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }


// ---- packed fp32x2 arithmetic (sm_100) and exp2 helpers -------------------
__device__ __forceinline__ uint64_t pk2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void up2(uint64_t r, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
// 2^x on the FMA pipe for x <= 0 (values below -126 flush to ~0):
// x = n + f with n = round(x), f in [-1/2, 1/2]; 2^f by a cubic fitted in
// relative error on Chebyshev nodes (max rel. error 7.8e-5, far below bf16's
// 3.9e-3); 2^n is added directly into the exponent field.
__device__ __forceinline__ uint64_t exp2_poly2(uint64_t x) {
  float a, b;
  up2(x, a, b);
  x = pk2(fmaxf(a, -126.f), fmaxf(b, -126.f));  // n >= -126 keeps the exponent sum >= 0
  const uint64_t magic = pk2(12582912.f, 12582912.f);  // 1.5 * 2^23: rounds to an integer
  const uint64_t t = add2(x, magic);
  const uint64_t n = add2(t, pk2(-12582912.f, -12582912.f));
  const uint64_t f = fma2(n, pk2(-1.f, -1.f), x);
  uint64_t q = fma2(pk2(0.05508868396f, 0.05508868396f), f, pk2(0.24260404706f, 0.24260404706f));
  q = fma2(q, f, pk2(0.69327622652f, 0.69327622652f));
  q = fma2(q, f, pk2(0.99992895126f, 0.99992895126f));
  float qa, qb, ta, tb;
  up2(q, qa, qb);
  up2(t, ta, tb);
  return pk2(__uint_as_float(__float_as_uint(qa) + (__float_as_uint(ta) << 23)),
             __uint_as_float(__float_as_uint(qb) + (__float_as_uint(tb) << 23)));
}
__device__ __forceinline__ uint64_t ex2_mufu2(uint64_t x) {
  float a, b;
  up2(x, a, b);
  return pk2(ex2(a), ex2(b));
}
__device__ __forceinline__ uint32_t pack_bf16x2_u64(uint64_t v) {
  float a, b;
  up2(v, a, b);
  return pack_bf16x2(a, b);
}

// Advance a shared-memory descriptor by a byte offset (the start-address field holds bytes >> 4
// and never carries: shared addresses stay below 2^18).  The base descriptor of a tile is built
// once and every K-step adds a compile-time constant, which keeps the single MMA-issuing thread
// from recomputing the whole descriptor per tcgen05.mma.
__device__ __forceinline__ uint64_t desc_add(uint64_t d, uint32_t bytes) { return d + (bytes >> 4); }

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// number of KV tiles visible to query tile [q0, q0+BM)
__device__ __forceinline__ int kv_tiles(const Params& p, int q0, int BN) {
  const int all = (p.Sk + BN - 1) / BN;
  if (!p.causal) return all;
  const int last_key = q0 + BM - 1 + (p.Sk - p.Sq);  // last key any row may see
  if (last_key < 0) return 0;
  const int t = last_key / BN + 1;
  return t < all ? t : all;
}

template <int DQK, int DV, int BN>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                    const __grid_constant__ CUtensorMap tv, Params p) {
  using C = Cfg<DQK, DV, BN>;
  static_assert(sizeof(Bars) <= 256, "Bars must fit its slot");
  extern __shared__ __align__(1024) uint8_t smem[];
  // The 128B-swizzle atoms assume 1024-byte aligned tiles; this kernel has no
  // static shared memory, so the dynamic base is the start of the CTA window.
  if (smem_u32(smem) & 1023) {
    if (threadIdx.x == 0) atomicCAS(&g_err, 0, 99);
    return;
  }
  Bars& bar = *reinterpret_cast<Bars*>(smem + C::BAR_OFF);
  float (*red_max)[2][BM] = reinterpret_cast<float (*)[2][BM]>(smem + C::RED_OFF);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  // heaviest (causal) tiles first
  // heaviest (causal) tiles first across the whole grid: CTAs launch in index order
  const int qt = p.num_qtiles - 1 - static_cast<int>(blockIdx.x / (p.B * p.H));
  const int bh = blockIdx.x % (p.B * p.H);
  const int h = bh % p.H, b = bh / p.H;
  const int hk = h / (p.H / p.Hk);
  const int q0 = qt * BM;
  const int nkv = kv_tiles(p, q0, BN);

  if (threadIdx.x == 0) {
    mbar_init(&bar.q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar.k_full[i], 1);
      mbar_init(&bar.v_full[i], 1);
      mbar_init(&bar.kv_empty[i], 1);
      mbar_init(&bar.s_full[i], 1);
      mbar_init(&bar.s_free[i], NUM_SM_WARPS);
      mbar_init(&bar.p_full[i], NUM_SM_WARPS);
      mbar_init(&bar.p_empty[i], 1);
      mbar_init(&bar.pv_full[i], 1);
      mbar_init(&bar.pv_free[i], NUM_SM_WARPS);
    }
    bar.abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tq);
    tma_prefetch_desc(&tk);
    tma_prefetch_desc(&tv);
  }
  if (warp == 1) tmem_alloc(&bar.tmem_base, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar.tmem_base;

  if (warp == 0) {
    if (lane == 0 && nkv > 0) {
      mbar_arrive_expect_tx(&bar.q_full, C::Q_BYTES);
#pragma unroll
      for (int c = 0; c < DQK / 64; ++c)
        tma_load_3d(smem + C::Q_OFF + c * (BM * 128), &tq, &bar.q_full, h * DQK + c * 64, q0, b);
      for (int j = 0; j < nkv; ++j) {
        const int st = j & 1;
        if (!mbar_wait(&bar.kv_empty[st], ((j >> 1) & 1) ^ 1, &bar.abort_flag, &g_err, 11)) break;
        const int k0 = j * BN;
        mbar_arrive_expect_tx(&bar.k_full[st], C::K_BYTES);
#pragma unroll
        for (int c = 0; c < DQK / 64; ++c)
          tma_load_3d(smem + C::K_OFF + st * C::K_BYTES + c * (BN * 128), &tk, &bar.k_full[st], hk * DQK + c * 64, k0,
                      b);
        mbar_arrive_expect_tx(&bar.v_full[st], C::V_BYTES);
#pragma unroll
        for (int c = 0; c < DV / 64; ++c)
          tma_load_3d(smem + C::V_OFF + st * C::V_BYTES + c * (BN * 128), &tv, &bar.v_full[st], hk * DV + c * 64, k0,
                      b);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && nkv > 0) {
      constexpr uint32_t idesc_s = umma_idesc_bf16(BM, BN, false, false);
      constexpr uint32_t idesc_pv = umma_idesc_bf16(BM, DV, false, true);
      const uint32_t q_addr = smem_u32(smem + C::Q_OFF);
      bool ok = mbar_wait(&bar.q_full, 0, &bar.abort_flag, &g_err, 12);
      auto issue_pv = [&](int i) -> bool {
        const int st = i & 1;
        if (!mbar_wait(&bar.v_full[st], (i >> 1) & 1, &bar.abort_flag, &g_err, 13)) return false;
        if (!mbar_wait(&bar.p_full[st], (i >> 1) & 1, &bar.abort_flag, &g_err, 14)) return false;
        if (!mbar_wait(&bar.pv_free[st], ((i >> 1) & 1) ^ 1, &bar.abort_flag, &g_err, 15)) return false;
        tc_fence_after();
        const uint32_t p_addr = smem_u32(smem + C::P_OFF + st * C::P_BYTES);
        const uint32_t v_addr = smem_u32(smem + C::V_OFF + st * C::V_BYTES);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint64_t ad = desc_add(umma_desc_sw128(p_addr, 16, 1024), (kk >> 2) * (BM * 128) + (kk & 3) * 32);
          const uint64_t bd = desc_add(umma_desc_sw128(v_addr, BN * 128, 1024), kk * 2048);
          umma_bf16(tmem + C::PV_COL + st * DV, ad, bd, idesc_pv, kk > 0 ? 1u : 0u);
        }
        umma_commit(&bar.pv_full[st]);
        umma_commit(&bar.kv_empty[st]);
        umma_commit(&bar.p_empty[st]);
        return true;
      };
      for (int j = 0; ok && j < nkv; ++j) {
        const int st = j & 1;
        if (!mbar_wait(&bar.k_full[st], (j >> 1) & 1, &bar.abort_flag, &g_err, 16)) break;
        if (!mbar_wait(&bar.s_free[st], ((j >> 1) & 1) ^ 1, &bar.abort_flag, &g_err, 17)) break;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(smem + C::K_OFF + st * C::K_BYTES);
#pragma unroll
        for (int kk = 0; kk < DQK / 16; ++kk) {
          const uint64_t ad = desc_add(umma_desc_sw128(q_addr, 16, 1024), (kk >> 2) * (BM * 128) + (kk & 3) * 32);
          const uint64_t bd = desc_add(umma_desc_sw128(k_addr, 16, 1024), (kk >> 2) * (BN * 128) + (kk & 3) * 32);
          umma_bf16(tmem + C::S_COL + st * BN, ad, bd, idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(&bar.s_full[st]);
        if (j > 0 && !issue_pv(j - 1)) {
          ok = false;
          break;
        }
      }
      if (ok) issue_pv(nkv - 1);
    }
  } else {
    // ---------------- softmax / output warps ----------------
    // Warp pair (w, w+4) shares TMEM lane quarter q (rows q*32..q*32+31);
    // half hh of the pair owns S columns [hh*HB, hh*HB+HB) and O columns
    // [hh*HD, hh*HD+HD).  Row maxima are exchanged through smem.
    constexpr int HB = BN / 2, HD = DV / 2;
    const int sw = warp - 2;
    const int q = warp & 3;
    const int hh = sw >> 2;
    const int r = q * 32 + lane;  // row within the tile (== TMEM lane)
    const int qrow = q0 + r;
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    const int diag = qrow + (p.Sk - p.Sq);  // last visible key for this row
    const float c2 = p.scale_log2;
    float o_acc[HD];
#pragma unroll
    for (int i = 0; i < HD; ++i) o_acc[i] = 0.f;
    float m_run = -INFINITY;   // running max (log2 domain, scaled) used for P_j
    float m_o = -INFINITY;     // normalisation of o_acc
    float l_run = 0.f;         // partial row sum over this warp's columns
    float m_prev = -INFINITY;  // max used for P_{j-1}
    bool ok = true;

    auto fold_pv = [&](int i, float m_i) -> bool {
      const int st = i & 1;
      if (!mbar_wait(&bar.pv_full[st], (i >> 1) & 1, &bar.abort_flag, &g_err, 21)) return false;
      tc_fence_after();
      const float alpha = (m_o == -INFINITY) ? 0.f : ex2(m_o - m_i);
      uint32_t v[HD];
#pragma unroll
      for (int c = 0; c < HD / 32; ++c)
        tmem_ld_32x32b_x32(tmem + lane_base + C::PV_COL + st * DV + hh * HD + c * 32,
                           *reinterpret_cast<uint32_t(*)[32]>(&v[c * 32]));
      tmem_ld_wait();
      const uint64_t al = pk2(alpha, alpha);
#pragma unroll
      for (int e = 0; e < HD; e += 2) {
        const uint64_t o = fma2(pk2(o_acc[e], o_acc[e + 1]), al, pk2(__uint_as_float(v[e]), __uint_as_float(v[e + 1])));
        up2(o, o_acc[e], o_acc[e + 1]);
      }
      m_o = m_i;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar.pv_free[st]);
      return true;
    };

    for (int j = 0; j < nkv; ++j) {
      const int st = j & 1;
      const int k0 = j * BN;
      if (!mbar_wait(&bar.s_full[st], (j >> 1) & 1, &bar.abort_flag, &g_err, 22)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sv[HB];
#pragma unroll
      for (int c = 0; c < HB / 32; ++c)
        tmem_ld_32x32b_x32(tmem + lane_base + C::S_COL + st * BN + hh * HB + c * 32,
                           *reinterpret_cast<uint32_t(*)[32]>(&sv[c * 32]));
      tmem_ld_wait();
      const int kbase = k0 + hh * HB;
      const bool need_mask = (p.causal && kbase + HB - 1 > q0 + (p.Sk - p.Sq)) || (kbase + HB > p.Sk);
      if (need_mask) {
#pragma unroll
        for (int e = 0; e < HB; ++e) {
          const int key = kbase + e;
          if (key >= p.Sk || (p.causal && key > diag)) sv[e] = __float_as_uint(-INFINITY);
        }
      }
      float mc[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int e = 0; e < HB; e += 8) {
#pragma unroll
        for (int u = 0; u < 4; ++u)
          mc[u] = max3(mc[u], __uint_as_float(sv[e + 2 * u]), __uint_as_float(sv[e + 2 * u + 1]));
      }
      float mx = max3(mc[0], mc[1], fmaxf(mc[2], mc[3]));
      red_max[st][hh][r] = mx;
      named_bar_sync(1 + q, 64);
      mx = fmaxf(mx, red_max[st][hh ^ 1][r]);
      const float m_new = fmaxf(m_run, mx * c2);
      const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
      // P_j buffer must be free (PV_{j-2} done)
      if (!mbar_wait(&bar.p_empty[st], ((j >> 1) & 1) ^ 1, &bar.abort_flag, &g_err, 23)) {
        ok = false;
        break;
      }
      uint8_t* rowp = smem + C::P_OFF + st * C::P_BYTES + ((hh * HB) / 64) * (BM * 128) + r * 128;
      const int chunk_base = ((hh * HB) % 64) / 8;
      const uint64_t cc = pk2(c2, c2), nm = pk2(-m_use, -m_use);
      uint64_t rs2 = pk2(0.f, 0.f);
#pragma unroll
      for (int u = 0; u < HB / 8; ++u) {
        uint32_t pk[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const uint64_t x = fma2(pk2(__uint_as_float(sv[u * 8 + 2 * e]), __uint_as_float(sv[u * 8 + 2 * e + 1])),
                                  cc, nm);
          // one pair in four goes to the FMA pipe so MUFU is not the limiter
          const uint64_t pv = (e == 3) ? exp2_poly2(x) : ex2_mufu2(x);
          rs2 = add2(rs2, pv);
          pk[e] = pack_bf16x2_u64(pv);
        }
        const int ch = (chunk_base + u) ^ (r & 7);
        *reinterpret_cast<uint4*>(rowp + ch * 16) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
      float rsa, rsb;
      up2(rs2, rsa, rsb);
      const float rs = rsa + rsb;
      // S buffer may be overwritten now; P is visible to the async proxy
      tc_fence_before();
      fence_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&bar.s_free[st]);
        mbar_arrive(&bar.p_full[st]);
      }
      const float alpha_l = (m_run == -INFINITY) ? 0.f : ex2(m_run - m_use);
      l_run = l_run * alpha_l + rs;
      m_run = m_new;
      if (j > 0 && !fold_pv(j - 1, m_prev)) {
        ok = false;
        break;
      }
      m_prev = m_use;
    }
    if (ok && nkv > 0) ok = fold_pv(nkv - 1, m_prev);
    // exchange partial row sums through the stage slot no tile of this row touches last
    float (*red_l)[BM] = red_max[nkv & 1];
    red_l[hh][r] = l_run;
    named_bar_sync(1 + q, 64);
    const float l_tot = red_l[0][r] + red_l[1][r];
    if (qrow < p.Sq) {
      const size_t row_off = ((static_cast<size_t>(b) * p.Sq + qrow) * p.H + h);
      __nv_bfloat16* orow = p.o + row_off * DV + hh * HD;
      const float inv = (ok && l_tot > 0.f) ? 1.f / l_tot : 0.f;
      // o_acc is normalised at m_o; l at m_run (equal unless trailing tiles were fully masked)
      const float fix = (m_o == -INFINITY || m_run == -INFINITY) ? 0.f : ex2(m_o - m_run) * inv;
#pragma unroll
      for (int c = 0; c < HD; c += 8) {
        uint4 w;
        w.x = pack_bf16x2(o_acc[c] * fix, o_acc[c + 1] * fix);
        w.y = pack_bf16x2(o_acc[c + 2] * fix, o_acc[c + 3] * fix);
        w.z = pack_bf16x2(o_acc[c + 4] * fix, o_acc[c + 5] * fix);
        w.w = pack_bf16x2(o_acc[c + 6] * fix, o_acc[c + 7] * fix);
        *reinterpret_cast<uint4*>(orow + c) = w;
      }
      if (hh == 0) {
        const float lse = (l_tot > 0.f && m_run != -INFINITY) ? (m_run + __log2f(l_tot)) * 0.69314718055994531f
                                                               : -INFINITY;
        p.lse[(static_cast<size_t>(b) * p.H + h) * lse_stride(p.Sq) + qrow] = lse;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// ============================================================================
// Forward, two query tiles per CTA (head dims 64/64 and 128/128).
//
// CTA = 256 queries of one head as tiles A (rows 0..127) and B (128..255)
// sharing every K/V tile.  TMEM (512 columns): tile t owns S_t (128 fp32
// columns, t*256) and O_t (DV fp32 columns, t*256+128).  The softmax warps
// of a tile (one per TMEM lane quarter, thread = query row) read S_t into
// registers, write P_t as packed bf16 back over the first 64 columns of S_t
// (tcgen05.st) and the PV MMA reads A = P_t straight from TMEM.  O_t stays
// in TMEM: it is rescaled only when a row's running max grows by more than
// 8 (log2 units), so P <= 256 and the rescale is rare.  While one tile's
// warps run softmax the tensor cores work on the other tile.
// Warps: 0 TMA producer, 1 MMA issuer, 2..5 softmax tile A, 6..9 tile B.
// ============================================================================
template <int DQK, int DV>
struct Cfg2 {
  static constexpr int BN = 128;
  static constexpr int Q_BYTES = BM * DQK * 2;  // per tile
  static constexpr int K_BYTES = BN * DQK * 2;
  static constexpr int V_BYTES = BN * DV * 2;
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = 2 * Q_BYTES;
  static constexpr int V_OFF = K_OFF + 2 * K_BYTES;
  static constexpr int BAR_OFF = V_OFF + 2 * V_BYTES;
  static constexpr int SMEM = BAR_OFF + 256;
  static_assert(DV <= 128, "O_t must fit next to S_t");
};

struct Bars2 {
  uint64_t q_full;
  uint64_t k_full[2], v_full[2], k_empty[2], v_empty[2];
  uint64_t s_full[2], p_full[2], pv_done[2];
  uint32_t tmem_base;
  int abort_flag;
};

__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
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
__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// D[tmem] (+)= A[tmem] * B[smem desc]
__device__ __forceinline__ void umma_bf16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

constexpr int FWD2_THREADS = 384;  // warpgroup 0: producer, MMA, 2 idle; warpgroups 1, 2: softmax

// 384 threads x 168 registers at launch >= 128 x (80 + 208 + 208): the softmax warpgroups hold
// a whole 128-column score row in registers
__device__ __forceinline__ void regs_dec_ctrl() { asm volatile("setmaxnreg.dec.sync.aligned.u32 80;"); }
__device__ __forceinline__ void regs_inc_softmax() { asm volatile("setmaxnreg.inc.sync.aligned.u32 208;"); }

template <int DQK, int DV>
__global__ void __launch_bounds__(FWD2_THREADS, 1)
    attn_fwd2_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                     const __grid_constant__ CUtensorMap tv, Params p) {
  using C = Cfg2<DQK, DV>;
  constexpr int BN = C::BN;
  extern __shared__ __align__(1024) uint8_t smem[];
  if (smem_u32(smem) & 1023) {
    if (threadIdx.x == 0) atomicCAS(&g_err, 0, 99);
    return;
  }
  Bars2& bar = *reinterpret_cast<Bars2*>(smem + C::BAR_OFF);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int npairs = (p.num_qtiles + 1) / 2;
  // heaviest pairs first across the whole grid (CTAs launch in index order)
  const int qp = npairs - 1 - static_cast<int>(blockIdx.x / (p.B * p.H));
  const int bh = blockIdx.x % (p.B * p.H);
  const int h = bh % p.H, b = bh / p.H;
  const int hk = h / (p.H / p.Hk);
  const int q0 = qp * 2 * BM;
  // KV tiles j0 .. j0 + nkv_t[t] - 1: with packed documents the pair starts at the document of
  // its first query (documents are contiguous, so later rows start no earlier)
  const int j0 = p.doc_start != nullptr ? p.doc_start[static_cast<size_t>(b) * p.Sq + q0] / BN : 0;
  int nkv_t[2];
  nkv_t[0] = max(kv_tiles(p, q0, BN) - j0, 0);
  nkv_t[1] = (q0 + BM < p.Sq) ? max(kv_tiles(p, q0 + BM, BN) - j0, 0) : 0;
  const int nkv = max(nkv_t[0], nkv_t[1]);

  if (threadIdx.x == 0) {
    mbar_init(&bar.q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar.k_full[i], 1);
      mbar_init(&bar.v_full[i], 1);
      mbar_init(&bar.k_empty[i], 1);
      mbar_init(&bar.v_empty[i], 1);
      mbar_init(&bar.s_full[i], 1);
      mbar_init(&bar.p_full[i], 4);
      mbar_init(&bar.pv_done[i], 1);
    }
    bar.abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tq);
    tma_prefetch_desc(&tk);
    tma_prefetch_desc(&tv);
  }
  if (warp == 1) tmem_alloc(&bar.tmem_base, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar.tmem_base;

  if (warp == 0) {
    regs_dec_ctrl();
    if (lane == 0 && nkv > 0) {
      mbar_arrive_expect_tx(&bar.q_full, 2 * C::Q_BYTES);
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int c = 0; c < DQK / 64; ++c)
          tma_load_3d(smem + C::Q_OFF + t * C::Q_BYTES + c * (BM * 128), &tq, &bar.q_full, h * DQK + c * 64,
                      q0 + t * BM, b);
      for (int j = 0; j < nkv; ++j) {
        const int st = j & 1;
        if (!mbar_wait(&bar.k_empty[st], ((j >> 1) & 1) ^ 1, &bar.abort_flag, &g_err, 51)) break;
        const int k0 = (j0 + j) * BN;
        mbar_arrive_expect_tx(&bar.k_full[st], C::K_BYTES);
#pragma unroll
        for (int c = 0; c < DQK / 64; ++c)
          tma_load_3d(smem + C::K_OFF + st * C::K_BYTES + c * (BN * 128), &tk, &bar.k_full[st], hk * DQK + c * 64, k0,
                      b);
        // K is released after the S MMAs, V only after PV: K of step j+2 streams in earlier
        if (!mbar_wait(&bar.v_empty[st], ((j >> 1) & 1) ^ 1, &bar.abort_flag, &g_err, 59)) break;
        mbar_arrive_expect_tx(&bar.v_full[st], C::V_BYTES);
#pragma unroll
        for (int c = 0; c < DV / 64; ++c)
          tma_load_3d(smem + C::V_OFF + st * C::V_BYTES + c * (BN * 128), &tv, &bar.v_full[st], hk * DV + c * 64, k0,
                      b);
      }
    }
  } else if (warp == 1) {
    regs_dec_ctrl();
    if (lane == 0 && nkv > 0) {
      constexpr uint32_t idesc_s = umma_idesc_bf16(BM, BN, false, false);
      constexpr uint32_t idesc_pv = umma_idesc_bf16(BM, DV, false, true);
      bool ok = mbar_wait(&bar.q_full, 0, &bar.abort_flag, &g_err, 52);
      // Ping-pong order: S_0(0) S_1(0) | PV_0(j) S_0(j+1) PV_1(j) S_1(j+1) | ...  While one
      // tile's softmax warps work on S_t(j+1), the tensor cores run the other tile's PV and S.
      // S_t(j+1) overwrites the columns PV_t(j) reads P_t(j) from; tcgen05.mma ops issued by
      // one thread execute in issue order, so the read precedes the overwrite.
      int k_ready = -1;
      auto need_k = [&](int j) -> bool {
        if (k_ready >= j) return true;
        k_ready = j;
        return mbar_wait(&bar.k_full[j & 1], (j >> 1) & 1, &bar.abort_flag, &g_err, 53);
      };
      auto issue_s = [&](int t, int j) {
        const uint32_t k_addr = smem_u32(smem + C::K_OFF + (j & 1) * C::K_BYTES);
        const uint32_t q_addr = smem_u32(smem + C::Q_OFF + t * C::Q_BYTES);
#pragma unroll
        for (int kk = 0; kk < DQK / 16; ++kk) {
          const uint64_t ad = desc_add(umma_desc_sw128(q_addr, 16, 1024), (kk >> 2) * (BM * 128) + (kk & 3) * 32);
          const uint64_t bd = desc_add(umma_desc_sw128(k_addr, 16, 1024), (kk >> 2) * (BN * 128) + (kk & 3) * 32);
          umma_bf16(tmem + t * 256, ad, bd, idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(&bar.s_full[t]);
      };
      if (ok) ok = need_k(0);
      if (ok) {
        tc_fence_after();
        for (int t = 0; t < 2; ++t)
          if (nkv_t[t] > 0) issue_s(t, 0);
        umma_commit(&bar.k_empty[0]);
      }
      for (int j = 0; ok && j < nkv; ++j) {
        const int st = j & 1;
        if (!mbar_wait(&bar.v_full[st], (j >> 1) & 1, &bar.abort_flag, &g_err, 55)) break;
        const uint32_t v_addr = smem_u32(smem + C::V_OFF + st * C::V_BYTES);
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          if (j >= nkv_t[t]) continue;
          if (!mbar_wait(&bar.p_full[t], j & 1, &bar.abort_flag, &g_err, 56)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk) {
            const uint64_t bd = desc_add(umma_desc_sw128(v_addr, BN * 128, 1024), kk * 2048);
            umma_bf16_ts(tmem + t * 256 + 128, tmem + t * 256 + kk * 8, bd, idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&bar.pv_done[t]);
          if (j + 1 < nkv_t[t]) {
            if (!need_k(j + 1)) { ok = false; break; }
            tc_fence_after();
            issue_s(t, j + 1);
          }
        }
        if (!ok) break;
        umma_commit(&bar.v_empty[st]);
        if (j + 1 < nkv) umma_commit(&bar.k_empty[(j + 1) & 1]);
      }
    }
  } else if (warp < 4) {
    regs_dec_ctrl();
  } else {
    regs_inc_softmax();
    const int t = (warp - 4) >> 2;  // query tile of this warp
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const int qrow = q0 + t * BM + r;
    const int nk = nkv_t[t];
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    const uint32_t s_col = tmem + lane_base + t * 256;
    const uint32_t o_col = s_col + 128;
    const int diag = qrow + (p.Sk - p.Sq);
    const int qt0 = q0 + t * BM;
    const int dstart = p.doc_start != nullptr ? p.doc_start[static_cast<size_t>(b) * p.Sq + min(qrow, p.Sq - 1)] : 0;
    const float c2 = p.scale_log2;
    float m_used = -INFINITY;  // max (log2 units) that P and O are currently normalised to
    float l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < nk; ++j) {
      if (!mbar_wait(&bar.s_full[t], j & 1, &bar.abort_flag, &g_err, 57)) { ok = false; break; }
      tc_fence_after();
      const int k0 = (j0 + j) * BN;
      const bool need_mask = (p.causal && k0 + BN - 1 > qt0 + (p.Sk - p.Sq)) || (k0 + BN > p.Sk);
      const int lo = dstart - k0;  // keys k0 + e with e < lo belong to earlier documents
      // S_t(j) row into registers once (four 32-column loads, one wait)
      uint32_t sv[BN];
#pragma unroll
      for (int c = 0; c < BN / 32; ++c)
        tmem_ld_32x32b_x32(s_col + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[c * 32]));
      tmem_ld_wait();
      if (need_mask || lo > 0) {  // keys k0 + e with e > lim are invisible (causal or past the end)
        const int lim = p.causal ? min(p.Sk - 1, diag) - k0 : p.Sk - 1 - k0;
#pragma unroll
        for (int e = 0; e < BN; ++e)
          if (e > lim || e < lo) sv[e] = __float_as_uint(-INFINITY);
      }
      float mc[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int e = 0; e < BN; e += 8) {
#pragma unroll
        for (int u = 0; u < 4; ++u)
          mc[u] = max3(mc[u], __uint_as_float(sv[e + 2 * u]), __uint_as_float(sv[e + 2 * u + 1]));
      }
      const float cand = max3(mc[0], mc[1], fmaxf(mc[2], mc[3])) * c2;
      // lazy rescale: only when the max grows by more than 8 (P stays <= 2^8)
      const bool grow = cand > (m_used == -INFINITY ? -INFINITY : m_used + 8.f);
      const bool rescale = __any_sync(0xffffffffu, grow);
      float alpha = 1.f;
      if (rescale) {
        const float m_new = fmaxf(m_used, cand);
        alpha = (m_used == -INFINITY || m_new == -INFINITY) ? 0.f : ex2(m_used - m_new);
        l_run *= alpha;
        m_used = m_new;
      }
      const float m_eff = (m_used == -INFINITY) ? 0.f : m_used;
      const uint64_t cc = pk2(c2, c2), nm = pk2(-m_eff, -m_eff);
      uint64_t rs2 = pk2(0.f, 0.f);
#pragma unroll
      for (int qq = 0; qq < 4; ++qq) {
        // P columns [qq*16, qq*16+16) hold keys [qq*32, qq*32+32) packed two per column
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const int ee = qq * 32 + e;
          const uint64_t x = fma2(pk2(__uint_as_float(sv[ee]), __uint_as_float(sv[ee + 1])), cc, nm);
          const uint64_t pv = ((e & 7) == 6) ? exp2_poly2(x) : ex2_mufu2(x);
          rs2 = add2(rs2, pv);
          pk[e / 2] = pack_bf16x2_u64(pv);
        }
        tmem_st_32x32b_x16(s_col + qq * 16, pk);
      }
      // O_t rescale after P is written (the scores are no longer live): PV_t(j) is issued only
      // after this warp's p_full arrival, and PV_t(j-1) is complete because S_t(j) is.
      if (rescale && j > 0) {
        const uint64_t al = pk2(alpha, alpha);
#pragma unroll 1
        for (int c = 0; c < DV / 32; ++c) {
          uint32_t ov[32];
          tmem_ld_32x32b_x32(o_col + c * 32, ov);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            float a0, a1;
            up2(mul2(pk2(__uint_as_float(ov[e]), __uint_as_float(ov[e + 1])), al), a0, a1);
            ov[e] = __float_as_uint(a0);
            ov[e + 1] = __float_as_uint(a1);
          }
          tmem_st_32x32b_x32(o_col + c * 32, ov);
        }
      }
      tmem_st_wait();
      float ra, rb;
      up2(rs2, ra, rb);
      l_run += ra + rb;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar.p_full[t]);
    }
    // final: wait for the last PV_t, normalise O_t and store
    bool have = ok && nk > 0 && mbar_wait(&bar.pv_done[t], (nk - 1) & 1, &bar.abort_flag, &g_err, 58);
    have = __all_sync(0xffffffffu, have);
    if (have) tc_fence_after();
    const float inv = (have && l_run > 0.f) ? 1.f / l_run : 0.f;
    const bool store = qrow < p.Sq;
    __nv_bfloat16* orow = p.o + ((static_cast<size_t>(b) * p.Sq + (store ? qrow : 0)) * p.H + h) * DV;
#pragma unroll
    for (int c = 0; c < DV / 32; ++c) {
      uint32_t ov[32];
      if (have) {
        tmem_ld_32x32b_x32(o_col + c * 32, ov);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) ov[e] = 0u;
      }
      if (store) {
#pragma unroll
        for (int e = 0; e < 32; e += 8)
          *reinterpret_cast<uint4*>(orow + c * 32 + e) =
              make_uint4(pack_bf16x2(__uint_as_float(ov[e]) * inv, __uint_as_float(ov[e + 1]) * inv),
                         pack_bf16x2(__uint_as_float(ov[e + 2]) * inv, __uint_as_float(ov[e + 3]) * inv),
                         pack_bf16x2(__uint_as_float(ov[e + 4]) * inv, __uint_as_float(ov[e + 5]) * inv),
                         pack_bf16x2(__uint_as_float(ov[e + 6]) * inv, __uint_as_float(ov[e + 7]) * inv));
      }
    }
    if (store) {
      const float lse = (l_run > 0.f && m_used != -INFINITY && have) ? (m_used + __log2f(l_run)) * 0.69314718055994531f
                                                                     : -INFINITY;
      p.lse[(static_cast<size_t>(b) * p.H + h) * lse_stride(p.Sq) + qrow] = lse;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int DQK, int DV>
void launch_fwd2(const void* q, const void* k, const void* v, Params& p, cudaStream_t s) {
  using C = Cfg2<DQK, DV>;
  static bool attr = false;
  auto* kern = attn_fwd2_kernel<DQK, DV>;
  if (!attr) {
    check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM), "attn2 smem");
    attr = true;
  }
  const CUtensorMap tq = make_tmap_bf16_3d(q, (uint64_t)p.H * DQK, p.Sq, p.B, (uint64_t)p.H * DQK,
                                           (uint64_t)p.Sq * p.H * DQK, 64, BM, 1);
  const CUtensorMap tk = make_tmap_bf16_3d(k, (uint64_t)p.Hk * DQK, p.Sk, p.B, (uint64_t)p.Hk * DQK,
                                           (uint64_t)p.Sk * p.Hk * DQK, 64, C::BN, 1);
  const CUtensorMap tv = make_tmap_bf16_3d(v, (uint64_t)p.Hk * DV, p.Sk, p.B, (uint64_t)p.Hk * DV,
                                           (uint64_t)p.Sk * p.Hk * DV, 64, C::BN, 1);
  const int grid = p.B * p.H * ((p.num_qtiles + 1) / 2);
  kern<<<grid, FWD2_THREADS, C::SMEM, s>>>(tq, tk, tv, p);
  check_cuda(cudaGetLastError(), "attn_fwd2 launch");
}

template <int DQK, int DV, int BN>
void launch_fwd(const void* q, const void* k, const void* v, Params& p, int Dqk, int Dv, cudaStream_t s) {
  using C = Cfg<DQK, DV, BN>;
  static bool attr = false;
  auto* kern = attn_fwd_kernel<DQK, DV, BN>;
  if (!attr) {
    check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM), "attn smem");
    attr = true;
  }
  const CUtensorMap tq = make_tmap_bf16_3d(q, (uint64_t)p.H * Dqk, p.Sq, p.B, (uint64_t)p.H * Dqk,
                                           (uint64_t)p.Sq * p.H * Dqk, 64, BM, 1);
  const CUtensorMap tk = make_tmap_bf16_3d(k, (uint64_t)p.Hk * Dqk, p.Sk, p.B, (uint64_t)p.Hk * Dqk,
                                           (uint64_t)p.Sk * p.Hk * Dqk, 64, BN, 1);
  const CUtensorMap tv = make_tmap_bf16_3d(v, (uint64_t)p.Hk * Dv, p.Sk, p.B, (uint64_t)p.Hk * Dv,
                                           (uint64_t)p.Sk * p.Hk * Dv, 64, BN, 1);
  const int grid = p.B * p.H * p.num_qtiles;
  kern<<<grid, NUM_THREADS, C::SMEM, s>>>(tq, tk, tv, p);
  check_cuda(cudaGetLastError(), "attn_fwd launch");
}


// ============================================================================
// Backward.
//   delta[b,h,q] = sum_d dO * O                                   (prep kernel)
//   dK/dV kernel: CTA = 128 keys of one KV head; iterates over the 64-query
//     tiles of every query head in the GQA group:
//       S^T = K Q^T, dP^T = V dO^T  (TMEM, double-buffered)
//       P^T = exp2(S^T*c - lse2), dS^T = P^T (dP^T - delta)    (softmax warps -> smem)
//       dV += P^T dO, dK += dS^T Q  (TMEM accumulators; no atomics)
//   dQ kernel: CTA = 128 queries of one head; iterates over 64-key tiles:
//       S = Q K^T, dP = dO V^T, dS = P (dP - delta), dQ += dS K
// ============================================================================

// delta = rowsum(dO * O) - dlse: a gradient flowing into the log-sum-exp output adds
// P * dlse to dS, i.e. shifts delta by -dlse (dlse laid out like lse; may be null)
__global__ void attn_bwd_delta_kernel(const __nv_bfloat16* __restrict__ dout, const __nv_bfloat16* __restrict__ o,
                                      float* __restrict__ delta, const float* __restrict__ dlse, int B, int S, int H,
                                      int Dv) {
  // one warp per (b, s, h) row
  const int64_t row = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  const int64_t rows = (int64_t)B * S * H;
  if (row >= rows) return;
  const __nv_bfloat16* a = dout + row * Dv;
  const __nv_bfloat16* c = o + row * Dv;
  float acc = 0.f;
  for (int d = lane * 2; d < Dv; d += 64) {
    const float2 x = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(a + d));
    const float2 y = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(c + d));
    acc += x.x * y.x + x.y * y.y;
  }
#pragma unroll
  for (int off = 16; off; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) {
    const int h = row % H;
    const int64_t bs = row / H;
    const int sidx = bs % S;
    const int bidx = bs / S;
    const int64_t at = ((int64_t)bidx * H + h) * lse_stride(S) + sidx;
    delta[at] = dlse != nullptr ? acc - dlse[at] : acc;
  }
}

struct BwdParams {
  int B, Sq, Sk, H, Hk;
  int causal;
  float scale;       // softmax scale
  float scale_log2;  // scale * log2(e)
  const float* lse;  // [B,H,Sq] natural log
  const float* delta;
  __nv_bfloat16* dk;
  __nv_bfloat16* dv;
  __nv_bfloat16* dq;
  const int* doc_start;  // as in Params (optional)
  const int* doc_end;
};


// element (r, c) of a [rows x 64] bf16 tile in the 128-byte-swizzled K-major layout
__device__ __forceinline__ void store_sw128_chunk(uint8_t* tile, int r, int chunk, uint4 v) {
  *reinterpret_cast<uint4*>(tile + r * 128 + ((chunk ^ (r & 7)) * 16)) = v;
}

template <int DQK, int DV, int NBUF>
struct DKVCfg {
  static constexpr int BK = 128;  // keys per CTA
  static constexpr int BQ = 64;   // queries per step
  static constexpr int K_BYTES = BK * DQK * 2;
  static constexpr int V_BYTES = BK * DV * 2;
  static constexpr int Q_BYTES = BQ * DQK * 2;
  static constexpr int O_BYTES = BQ * DV * 2;  // dO tile
  static constexpr int K_OFF = 0;
  static constexpr int V_OFF = K_OFF + K_BYTES;
  static constexpr int Q_OFF = V_OFF + V_BYTES;
  // Q/dO ring depth: P^T and dS^T live in TMEM, so shared memory goes to prefetch
  static constexpr int QS = (DQK > 128) ? 3 : (DQK > 64 ? 4 : 6);
  static constexpr int DO_OFF = Q_OFF + QS * Q_BYTES;
  static constexpr int SMEM = DO_OFF + QS * O_BYTES + 1024;
  static constexpr int ST_COL = 0;                 // NBUF x BQ
  static constexpr int DPT_COL = NBUF * BQ;        // NBUF x BQ
  static constexpr int DV_COL = 2 * NBUF * BQ;     // DV
  static constexpr int DK_COL = DV_COL + DV;       // DQK
  static_assert(DK_COL + DQK <= 512, "TMEM budget");
};

constexpr int kMaxQS = 6;
struct DKVBars {
  uint64_t kv_full;
  uint64_t qd_full[kMaxQS], qd_empty[kMaxQS];
  uint64_t s_full[2], s_free[2];
  uint64_t p_full[2];
  uint64_t acc_full;
  uint32_t tmem_base;
  int abort_flag;
  alignas(16) float lse2[kMaxQS][64];  // lse (natural log) of the staged 64 queries (bulk-copied)
  alignas(16) float dlt[kMaxQS][64];   // delta of the staged 64 queries (bulk-copied)
};

template <int DQK, int DV, int NBUF>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    attn_bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tdo,
                         const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv, BwdParams p) {
  using C = DKVCfg<DQK, DV, NBUF>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ DKVBars bar;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int nkt = (p.Sk + C::BK - 1) / C::BK;
  // under a causal mask the first key tiles see the most queries: launch them first, grid-wide
  const int kt = blockIdx.x / (p.B * p.Hk);
  const int bhk = blockIdx.x % (p.B * p.Hk);
  const int hk = bhk % p.Hk, b = bhk / p.Hk;
  const int group = p.H / p.Hk;
  const int k0 = kt * C::BK;
  const int offset = p.Sk - p.Sq;
  const int nqt = (p.Sq + C::BQ - 1) / C::BQ;
  int qt_first = 0;
  if (p.causal) {
    const int first_q = k0 - offset;  // smallest query that sees key k0
    qt_first = first_q <= 0 ? 0 : first_q / C::BQ;
  }
  int qt_last = nqt - 1;
  if (p.doc_end != nullptr) {  // no query past the end of the last key's document sees this tile
    const int kl = min(k0 + C::BK, p.Sk) - 1;
    qt_last = min(qt_last, (p.doc_end[static_cast<size_t>(b) * p.Sk + kl] - 1) / C::BQ);
  }
  const int per_head = qt_last >= qt_first ? qt_last - qt_first + 1 : 0;
  const int items = per_head * group;

  if (threadIdx.x == 0) {
    mbar_init(&bar.kv_full, 1);
    static_assert(C::QS <= kMaxQS, "Q/dO ring");
    for (int i = 0; i < C::QS; ++i) {
      mbar_init(&bar.qd_full[i], 1);
      mbar_init(&bar.qd_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar.s_full[i], 1);
      mbar_init(&bar.s_free[i], NUM_SM_WARPS);
      mbar_init(&bar.p_full[i], NUM_SM_WARPS);
    }
    mbar_init(&bar.acc_full, 1);
    bar.abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tq);
    tma_prefetch_desc(&tdo);
    tma_prefetch_desc(&tk);
    tma_prefetch_desc(&tv);
  }
  if (warp == 1) tmem_alloc(&bar.tmem_base, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar.tmem_base;

  if (warp == 0) {
    if (lane == 0 && items > 0) {
      mbar_arrive_expect_tx(&bar.kv_full, C::K_BYTES + C::V_BYTES);
#pragma unroll
      for (int c = 0; c < DQK / 64; ++c)
        tma_load_3d(smem + C::K_OFF + c * (C::BK * 128), &tk, &bar.kv_full, hk * DQK + c * 64, k0, b);
#pragma unroll
      for (int c = 0; c < DV / 64; ++c)
        tma_load_3d(smem + C::V_OFF + c * (C::BK * 128), &tv, &bar.kv_full, hk * DV + c * 64, k0, b);
      for (int i = 0; i < items; ++i) {
        const int st = i % C::QS;
        const int h = hk * group + i / per_head;
        const int q0 = (qt_first + i % per_head) * C::BQ;
        if (!mbar_wait(&bar.qd_empty[st], ((i / C::QS) & 1) ^ 1, &bar.abort_flag, &g_err, 31)) break;
        mbar_arrive_expect_tx(&bar.qd_full[st], C::Q_BYTES + C::O_BYTES + 2 * 64 * 4);
        const size_t row = ((size_t)b * p.H + h) * lse_stride(p.Sq) + q0;
        bulk_copy_g2s(&bar.lse2[st][0], p.lse + row, 256, &bar.qd_full[st]);
        bulk_copy_g2s(&bar.dlt[st][0], p.delta + row, 256, &bar.qd_full[st]);
#pragma unroll
        for (int c = 0; c < DQK / 64; ++c)
          tma_load_3d(smem + C::Q_OFF + st * C::Q_BYTES + c * (C::BQ * 128), &tq, &bar.qd_full[st], h * DQK + c * 64,
                      q0, b);
#pragma unroll
        for (int c = 0; c < DV / 64; ++c)
          tma_load_3d(smem + C::DO_OFF + st * C::O_BYTES + c * (C::BQ * 128), &tdo, &bar.qd_full[st], h * DV + c * 64,
                      q0, b);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && items > 0) {
      constexpr uint32_t idesc_s = umma_idesc_bf16(C::BK, C::BQ, false, false);   // S^T, dP^T
      constexpr uint32_t idesc_dv = umma_idesc_bf16(C::BK, DV, false, true);      // dV += P^T dO
      constexpr uint32_t idesc_dk = umma_idesc_bf16(C::BK, DQK, false, true);     // dK += dS^T Q
      const uint32_t k_addr = smem_u32(smem + C::K_OFF), v_addr = smem_u32(smem + C::V_OFF);
      bool ok = mbar_wait(&bar.kv_full, 0, &bar.abort_flag, &g_err, 32);
      // P^T and dS^T come from TMEM (packed bf16 written by the softmax warps over the columns of
      // S^T and dP^T they read): queries [32h, 32h+32) of buffer sb sit at columns 32h..32h+15.
      auto issue_grads = [&](int i) -> bool {
        const int st = i & 1;
        const int sb = i % NBUF;
        if (!mbar_wait(&bar.p_full[st], (i >> 1) & 1, &bar.abort_flag, &g_err, 33)) return false;
        tc_fence_after();
        const int qs = i % C::QS;
        const uint32_t qa = smem_u32(smem + C::Q_OFF + qs * C::Q_BYTES);
        const uint32_t da = smem_u32(smem + C::DO_OFF + qs * C::O_BYTES);
        const uint32_t pt = tmem + C::ST_COL + sb * C::BQ, dst = tmem + C::DPT_COL + sb * C::BQ;
#pragma unroll
        for (int kk = 0; kk < C::BQ / 16; ++kk) {
          const uint64_t b1 = desc_add(umma_desc_sw128(da, C::BQ * 128, 1024), kk * 2048);
          umma_bf16_ts(tmem + C::DV_COL, pt + (kk >> 1) * 32 + (kk & 1) * 8, b1, idesc_dv, (i > 0 || kk > 0) ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < C::BQ / 16; ++kk) {
          const uint64_t b2 = desc_add(umma_desc_sw128(qa, C::BQ * 128, 1024), kk * 2048);
          umma_bf16_ts(tmem + C::DK_COL, dst + (kk >> 1) * 32 + (kk & 1) * 8, b2, idesc_dk, (i > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&bar.qd_empty[qs]);
        return true;
      };
      for (int i = 0; ok && i < items; ++i) {
        const int qs = i % C::QS;
        const int sb = i % NBUF;
        if (!mbar_wait(&bar.qd_full[qs], (i / C::QS) & 1, &bar.abort_flag, &g_err, 34)) { ok = false; break; }
        // one S/dP buffer: the gradient MMAs of step i-1 read P/dS from it, so they go first
        // (tcgen05.mma ops of one thread execute in issue order)
        if (NBUF == 1 && i > 0 && !issue_grads(i - 1)) { ok = false; break; }
        if (!mbar_wait(&bar.s_free[sb], ((i / NBUF) & 1) ^ 1, &bar.abort_flag, &g_err, 35)) { ok = false; break; }
        tc_fence_after();
        const uint32_t qa = smem_u32(smem + C::Q_OFF + qs * C::Q_BYTES);
        const uint32_t da = smem_u32(smem + C::DO_OFF + qs * C::O_BYTES);
#pragma unroll
        for (int kk = 0; kk < DQK / 16; ++kk) {
          const uint64_t a = desc_add(umma_desc_sw128(k_addr, 16, 1024), (kk >> 2) * (C::BK * 128) + (kk & 3) * 32);
          const uint64_t bq = desc_add(umma_desc_sw128(qa, 16, 1024), (kk >> 2) * (C::BQ * 128) + (kk & 3) * 32);
          umma_bf16(tmem + C::ST_COL + sb * C::BQ, a, bq, idesc_s, kk > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < DV / 16; ++kk) {
          const uint64_t a = desc_add(umma_desc_sw128(v_addr, 16, 1024), (kk >> 2) * (C::BK * 128) + (kk & 3) * 32);
          const uint64_t bo = desc_add(umma_desc_sw128(da, 16, 1024), (kk >> 2) * (C::BQ * 128) + (kk & 3) * 32);
          umma_bf16(tmem + C::DPT_COL + sb * C::BQ, a, bo, idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(&bar.s_full[sb]);
        // two buffers: the softmax of step i overlaps the gradient MMAs of step i-1
        if (NBUF == 2 && i > 0 && !issue_grads(i - 1)) { ok = false; break; }
      }
      if (ok) ok = issue_grads(items - 1);
      if (ok) umma_commit(&bar.acc_full);
    }
  } else {
    const int q = warp & 3;
    const int hh = (warp - 2) >> 2;  // which 32-query half of the tile this warp handles
    const int r = q * 32 + lane;     // key row within the tile
    const int kidx = k0 + r;
    const int dend = p.doc_end != nullptr ? p.doc_end[static_cast<size_t>(b) * p.Sk + min(kidx, p.Sk - 1)] : 0x7fffffff;
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    bool ok = true;
    for (int i = 0; i < items; ++i) {
      const int st = i & 1;
      const int sb = i % NBUF;
      const int h = hk * group + i / per_head;
      const int q0 = (qt_first + i % per_head) * C::BQ;
      // lse / delta of this query tile arrive with the Q/dO tiles
      const int qs = i % C::QS;
      if (!mbar_wait(&bar.qd_full[qs], (i / C::QS) & 1, &bar.abort_flag, &g_err, 39)) { ok = false; break; }
      // S(i) complete implies the gradient MMAs of step i - NBUF (which read this buffer's P/dS)
      // are complete too: they were issued before it
      if (!mbar_wait(&bar.s_full[sb], (i / NBUF) & 1, &bar.abort_flag, &g_err, 36)) { ok = false; break; }
      tc_fence_after();
      const bool need_mask = (kidx >= p.Sk) || (q0 + C::BQ > p.Sq) || (p.causal && k0 + C::BK - 1 > q0 + offset) ||
                             (q0 + C::BQ > dend);
      {
        const int c = hh;
        uint32_t sv[32], dv[32];
        tmem_ld_32x32b_x32(tmem + lane_base + C::ST_COL + sb * C::BQ + c * 32, sv);
        tmem_ld_32x32b_x32(tmem + lane_base + C::DPT_COL + sb * C::BQ + c * 32, dv);
        tmem_ld_wait();
        uint32_t pk[16], dk[16];
        const uint64_t cc = pk2(p.scale_log2, p.scale_log2);
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const int col = c * 32 + e;
          const float2 ls = *reinterpret_cast<const float2*>(&bar.lse2[qs][col]);
          const float2 dl = *reinterpret_cast<const float2*>(&bar.dlt[qs][col]);
          const uint64_t nl = mul2(pk2(ls.x, ls.y), pk2(-1.4426950408889634f, -1.4426950408889634f));
          const uint64_t x = fma2(pk2(__uint_as_float(sv[e]), __uint_as_float(sv[e + 1])), cc, nl);
          uint64_t pv = ((e & 7) == 6) ? exp2_poly2(x) : ex2_mufu2(x);
          if (need_mask) {
            float a0, a1;
            up2(pv, a0, a1);
            const int qi = q0 + col;
            if (kidx >= p.Sk || qi >= p.Sq || qi >= dend || (p.causal && kidx > qi + offset)) a0 = 0.f;
            if (kidx >= p.Sk || qi + 1 >= p.Sq || qi + 1 >= dend || (p.causal && kidx > qi + 1 + offset)) a1 = 0.f;
            pv = pk2(a0, a1);
          }
          const uint64_t ds = mul2(pv, add2(pk2(__uint_as_float(dv[e]), __uint_as_float(dv[e + 1])), pk2(-dl.x, -dl.y)));
          pk[e / 2] = pack_bf16x2_u64(pv);
          dk[e / 2] = pack_bf16x2_u64(ds);
        }
        // packed over the first half of the columns this warp just read
        tmem_st_32x32b_x16(tmem + lane_base + C::ST_COL + sb * C::BQ + c * 32, pk);
        tmem_st_32x32b_x16(tmem + lane_base + C::DPT_COL + sb * C::BQ + c * 32, dk);
        tmem_st_wait();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&bar.s_free[sb]);
        mbar_arrive(&bar.p_full[st]);
      }
    }
    // epilogue: dV, dK rows (TMEM loads are warp-collective: every lane loads, valid rows store)
    bool have = ok && items > 0 && mbar_wait(&bar.acc_full, 0, &bar.abort_flag, &g_err, 38);
    have = __all_sync(0xffffffffu, have);
    if (have) tc_fence_after();
    const bool store = kidx < p.Sk;
    const size_t row = ((size_t)b * p.Sk + (store ? kidx : 0)) * p.Hk + hk;
    __nv_bfloat16* dvrow = p.dv + row * DV;
    __nv_bfloat16* dkrow = p.dk + row * DQK;
#pragma unroll 1
    for (int c = hh; c < (DV + DQK) / 32; c += 2) {
      uint32_t v[32];
      if (have) {
        tmem_ld_32x32b_x32(tmem + lane_base + C::DV_COL + c * 32, v);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) v[e] = 0u;
      }
      const bool is_dv = c < DV / 32;
      const float sc = is_dv ? 1.f : p.scale;
      __nv_bfloat16* dstp = is_dv ? dvrow + c * 32 : dkrow + (c - DV / 32) * 32;
      if (store) {
#pragma unroll
        for (int e = 0; e < 32; e += 8)
          *reinterpret_cast<uint4*>(dstp + e) =
              make_uint4(pack_bf16x2(__uint_as_float(v[e]) * sc, __uint_as_float(v[e + 1]) * sc),
                         pack_bf16x2(__uint_as_float(v[e + 2]) * sc, __uint_as_float(v[e + 3]) * sc),
                         pack_bf16x2(__uint_as_float(v[e + 4]) * sc, __uint_as_float(v[e + 5]) * sc),
                         pack_bf16x2(__uint_as_float(v[e + 6]) * sc, __uint_as_float(v[e + 7]) * sc));
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int DQK, int DV>
struct DQCfg {
  static constexpr int BQ = 128;  // queries per CTA
  static constexpr int BK = 64;   // keys per step
  static constexpr int Q_BYTES = BQ * DQK * 2;
  static constexpr int O_BYTES = BQ * DV * 2;
  static constexpr int K_BYTES = BK * DQK * 2;
  static constexpr int V_BYTES = BK * DV * 2;
  static constexpr int Q_OFF = 0;
  static constexpr int DO_OFF = Q_OFF + Q_BYTES;
  static constexpr int K_OFF = DO_OFF + O_BYTES;
  // K/V ring depth (dS lives in TMEM, so shared memory goes to prefetch)
  static constexpr int KS = (DQK > 128) ? 3 : (DQK > 64 ? 5 : 6);
  static constexpr int V_OFF = K_OFF + KS * K_BYTES;
  static constexpr int SMEM = V_OFF + KS * V_BYTES + 1024;
  static constexpr int S_COL = 0;          // 2 x BK
  static constexpr int DP_COL = 2 * BK;    // 2 x BK
  static constexpr int DQ_COL = 4 * BK;    // DQK
  static_assert(DQ_COL + DQK <= 512, "TMEM budget");
};

struct DQBars {
  uint64_t qd_full;
  uint64_t kv_full[6], kv_empty[6];
  uint64_t s_full[2], s_free[2];
  uint64_t ds_full[2];
  uint64_t acc_full;
  uint32_t tmem_base;
  int abort_flag;
};

template <int DQK, int DV>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    attn_bwd_dq_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tdo,
                       const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv, BwdParams p) {
  using C = DQCfg<DQK, DV>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ DQBars bar;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int nqt = (p.Sq + C::BQ - 1) / C::BQ;
  const int qt = nqt - 1 - static_cast<int>(blockIdx.x / (p.B * p.H));  // heaviest first, grid-wide
  const int bh = blockIdx.x % (p.B * p.H);
  const int h = bh % p.H, b = bh / p.H;
  const int hk = h / (p.H / p.Hk);
  const int q0 = qt * C::BQ;
  const int offset = p.Sk - p.Sq;
  int nkv = (p.Sk + C::BK - 1) / C::BK;
  if (p.causal) {
    const int last_key = q0 + C::BQ - 1 + offset;
    nkv = last_key < 0 ? 0 : min(nkv, last_key / C::BK + 1);
  }
  // packed documents: key tiles start at the document of the tile's first query
  const int j0 = p.doc_start != nullptr ? p.doc_start[static_cast<size_t>(b) * p.Sq + q0] / C::BK : 0;
  nkv = max(nkv - j0, 0);

  if (threadIdx.x == 0) {
    mbar_init(&bar.qd_full, 1);
    static_assert(C::KS <= 6, "K/V ring");
    for (int i = 0; i < C::KS; ++i) {
      mbar_init(&bar.kv_full[i], 1);
      mbar_init(&bar.kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar.s_full[i], 1);
      mbar_init(&bar.s_free[i], NUM_SM_WARPS);
      mbar_init(&bar.ds_full[i], NUM_SM_WARPS);
    }
    mbar_init(&bar.acc_full, 1);
    bar.abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tq);
    tma_prefetch_desc(&tdo);
    tma_prefetch_desc(&tk);
    tma_prefetch_desc(&tv);
  }
  if (warp == 1) tmem_alloc(&bar.tmem_base, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar.tmem_base;

  if (warp == 0) {
    if (lane == 0 && nkv > 0) {
      mbar_arrive_expect_tx(&bar.qd_full, C::Q_BYTES + C::O_BYTES);
#pragma unroll
      for (int c = 0; c < DQK / 64; ++c)
        tma_load_3d(smem + C::Q_OFF + c * (C::BQ * 128), &tq, &bar.qd_full, h * DQK + c * 64, q0, b);
#pragma unroll
      for (int c = 0; c < DV / 64; ++c)
        tma_load_3d(smem + C::DO_OFF + c * (C::BQ * 128), &tdo, &bar.qd_full, h * DV + c * 64, q0, b);
      for (int j = 0; j < nkv; ++j) {
        const int st = j % C::KS;
        if (!mbar_wait(&bar.kv_empty[st], ((j / C::KS) & 1) ^ 1, &bar.abort_flag, &g_err, 41)) break;
        mbar_arrive_expect_tx(&bar.kv_full[st], C::K_BYTES + C::V_BYTES);
#pragma unroll
        for (int c = 0; c < DQK / 64; ++c)
          tma_load_3d(smem + C::K_OFF + st * C::K_BYTES + c * (C::BK * 128), &tk, &bar.kv_full[st], hk * DQK + c * 64,
                      (j0 + j) * C::BK, b);
#pragma unroll
        for (int c = 0; c < DV / 64; ++c)
          tma_load_3d(smem + C::V_OFF + st * C::V_BYTES + c * (C::BK * 128), &tv, &bar.kv_full[st], hk * DV + c * 64,
                      (j0 + j) * C::BK, b);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && nkv > 0) {
      constexpr uint32_t idesc_s = umma_idesc_bf16(C::BQ, C::BK, false, false);
      constexpr uint32_t idesc_dq = umma_idesc_bf16(C::BQ, DQK, false, true);
      const uint32_t qa = smem_u32(smem + C::Q_OFF), da = smem_u32(smem + C::DO_OFF);
      bool ok = mbar_wait(&bar.qd_full, 0, &bar.abort_flag, &g_err, 42);
      auto issue_dq = [&](int i) -> bool {
        const int st = i & 1;
        if (!mbar_wait(&bar.ds_full[st], (i >> 1) & 1, &bar.abort_flag, &g_err, 43)) return false;
        tc_fence_after();
        const int ks = i % C::KS;
        // dS from TMEM: keys [32h, 32h+32) of buffer st packed at columns 32h..32h+15
        const uint32_t ds = tmem + C::S_COL + st * C::BK;
        const uint32_t ka = smem_u32(smem + C::K_OFF + ks * C::K_BYTES);
#pragma unroll
        for (int kk = 0; kk < C::BK / 16; ++kk) {
          const uint64_t bb = desc_add(umma_desc_sw128(ka, C::BK * 128, 1024), kk * 2048);
          umma_bf16_ts(tmem + C::DQ_COL, ds + (kk >> 1) * 32 + (kk & 1) * 8, bb, idesc_dq, (i > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&bar.kv_empty[ks]);
        return true;
      };
      for (int j = 0; ok && j < nkv; ++j) {
        const int st = j & 1;
        const int ks = j % C::KS;
        if (!mbar_wait(&bar.kv_full[ks], (j / C::KS) & 1, &bar.abort_flag, &g_err, 44)) { ok = false; break; }
        if (!mbar_wait(&bar.s_free[st], ((j >> 1) & 1) ^ 1, &bar.abort_flag, &g_err, 45)) { ok = false; break; }
        tc_fence_after();
        const uint32_t ka = smem_u32(smem + C::K_OFF + ks * C::K_BYTES);
        const uint32_t va = smem_u32(smem + C::V_OFF + ks * C::V_BYTES);
#pragma unroll
        for (int kk = 0; kk < DQK / 16; ++kk) {
          const uint64_t a = desc_add(umma_desc_sw128(qa, 16, 1024), (kk >> 2) * (C::BQ * 128) + (kk & 3) * 32);
          const uint64_t bb = desc_add(umma_desc_sw128(ka, 16, 1024), (kk >> 2) * (C::BK * 128) + (kk & 3) * 32);
          umma_bf16(tmem + C::S_COL + st * C::BK, a, bb, idesc_s, kk > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < DV / 16; ++kk) {
          const uint64_t a = desc_add(umma_desc_sw128(da, 16, 1024), (kk >> 2) * (C::BQ * 128) + (kk & 3) * 32);
          const uint64_t bb = desc_add(umma_desc_sw128(va, 16, 1024), (kk >> 2) * (C::BK * 128) + (kk & 3) * 32);
          umma_bf16(tmem + C::DP_COL + st * C::BK, a, bb, idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(&bar.s_full[st]);
        if (j > 0 && !issue_dq(j - 1)) { ok = false; break; }
      }
      if (ok) ok = issue_dq(nkv - 1);
      if (ok) umma_commit(&bar.acc_full);
    }
  } else {
    const int q = warp & 3;
    const int hh = (warp - 2) >> 2;  // which 32-key half of each tile this warp handles
    const int r = q * 32 + lane;
    const int qi = q0 + r;
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    const bool qvalid = qi < p.Sq;
    const float lse2 = qvalid ? p.lse[((size_t)b * p.H + h) * lse_stride(p.Sq) + qi] * 1.4426950408889634f : INFINITY;
    const float dl = qvalid ? p.delta[((size_t)b * p.H + h) * lse_stride(p.Sq) + qi] : 0.f;
    const int diag = qi + offset;
    const int dstart = p.doc_start != nullptr ? p.doc_start[static_cast<size_t>(b) * p.Sq + min(qi, p.Sq - 1)] : 0;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      const int st = j & 1;
      const int k0 = (j0 + j) * C::BK;
      if (!mbar_wait(&bar.s_full[st], (j >> 1) & 1, &bar.abort_flag, &g_err, 46)) { ok = false; break; }
      // S(j) complete implies dQ(j-2), which read dS(j-2) from this buffer, is complete
      tc_fence_after();
      const bool need_mask = !qvalid || (k0 + C::BK > p.Sk) || (p.causal && k0 + C::BK - 1 > diag) || (k0 < dstart);
      {
        const int c = hh;
        uint32_t sv[32], dv[32];
        tmem_ld_32x32b_x32(tmem + lane_base + C::S_COL + st * C::BK + c * 32, sv);
        tmem_ld_32x32b_x32(tmem + lane_base + C::DP_COL + st * C::BK + c * 32, dv);
        tmem_ld_wait();
        uint32_t pk[16];
        const uint64_t cc = pk2(p.scale_log2, p.scale_log2), nl = pk2(-lse2, -lse2), nd = pk2(-dl, -dl);
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const uint64_t x = fma2(pk2(__uint_as_float(sv[e]), __uint_as_float(sv[e + 1])), cc, nl);
          uint64_t pv = ((e & 7) == 6) ? exp2_poly2(x) : ex2_mufu2(x);
          if (need_mask) {
            float a0, a1;
            up2(pv, a0, a1);
            const int key = k0 + c * 32 + e;
            if (!qvalid || key >= p.Sk || key < dstart || (p.causal && key > diag)) a0 = 0.f;
            if (!qvalid || key + 1 >= p.Sk || key + 1 < dstart || (p.causal && key + 1 > diag)) a1 = 0.f;
            pv = pk2(a0, a1);
          }
          pk[e / 2] = pack_bf16x2_u64(mul2(pv, add2(pk2(__uint_as_float(dv[e]), __uint_as_float(dv[e + 1])), nd)));
        }
        tmem_st_32x32b_x16(tmem + lane_base + C::S_COL + st * C::BK + c * 32, pk);  // over what it read
        tmem_st_wait();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&bar.s_free[st]);
        mbar_arrive(&bar.ds_full[st]);
      }
    }
    bool have = ok && nkv > 0 && mbar_wait(&bar.acc_full, 0, &bar.abort_flag, &g_err, 48);
    have = __all_sync(0xffffffffu, have);
    if (have) tc_fence_after();
    __nv_bfloat16* dqrow = p.dq + (((size_t)b * p.Sq + (qvalid ? qi : 0)) * p.H + h) * DQK;
#pragma unroll 1
    for (int c = hh; c < DQK / 32; c += 2) {
      uint32_t v[32];
      if (have) {
        tmem_ld_32x32b_x32(tmem + lane_base + C::DQ_COL + c * 32, v);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) v[e] = 0u;
      }
      const float sc = p.scale;
      if (qvalid) {
#pragma unroll
        for (int e = 0; e < 32; e += 8)
          *reinterpret_cast<uint4*>(dqrow + c * 32 + e) =
              make_uint4(pack_bf16x2(__uint_as_float(v[e]) * sc, __uint_as_float(v[e + 1]) * sc),
                         pack_bf16x2(__uint_as_float(v[e + 2]) * sc, __uint_as_float(v[e + 3]) * sc),
                         pack_bf16x2(__uint_as_float(v[e + 4]) * sc, __uint_as_float(v[e + 5]) * sc),
                         pack_bf16x2(__uint_as_float(v[e + 6]) * sc, __uint_as_float(v[e + 7]) * sc));
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int DQK, int DV, int NBUF>
void launch_bwd(const void* dout, const void* q, const void* k, const void* v, BwdParams& p, cudaStream_t s) {
  using CK = DKVCfg<DQK, DV, NBUF>;
  using CQ = DQCfg<DQK, DV>;
  static bool attr = false;
  auto* kdkv = attn_bwd_dkdv_kernel<DQK, DV, NBUF>;
  auto* kdq = attn_bwd_dq_kernel<DQK, DV>;
  if (!attr) {
    check_cuda(cudaFuncSetAttribute(kdkv, cudaFuncAttributeMaxDynamicSharedMemorySize, CK::SMEM), "attn bwd smem");
    check_cuda(cudaFuncSetAttribute(kdq, cudaFuncAttributeMaxDynamicSharedMemorySize, CQ::SMEM), "attn bwd smem");
    attr = true;
  }
  const uint64_t qs = (uint64_t)p.H * DQK, os = (uint64_t)p.H * DV, ks = (uint64_t)p.Hk * DQK, vs = (uint64_t)p.Hk * DV;
  // dK/dV kernel: 64-query tiles, 128-key tiles
  {
    const CUtensorMap tq = make_tmap_bf16_3d(q, qs, p.Sq, p.B, qs, qs * p.Sq, 64, CK::BQ, 1);
    const CUtensorMap tdo = make_tmap_bf16_3d(dout, os, p.Sq, p.B, os, os * p.Sq, 64, CK::BQ, 1);
    const CUtensorMap tk = make_tmap_bf16_3d(k, ks, p.Sk, p.B, ks, ks * p.Sk, 64, CK::BK, 1);
    const CUtensorMap tv = make_tmap_bf16_3d(v, vs, p.Sk, p.B, vs, vs * p.Sk, 64, CK::BK, 1);
    const int grid = p.B * p.Hk * ((p.Sk + CK::BK - 1) / CK::BK);
    kdkv<<<grid, NUM_THREADS, CK::SMEM, s>>>(tq, tdo, tk, tv, p);
    check_cuda(cudaGetLastError(), "attn_bwd_dkdv launch");
  }
  {
    const CUtensorMap tq = make_tmap_bf16_3d(q, qs, p.Sq, p.B, qs, qs * p.Sq, 64, CQ::BQ, 1);
    const CUtensorMap tdo = make_tmap_bf16_3d(dout, os, p.Sq, p.B, os, os * p.Sq, 64, CQ::BQ, 1);
    const CUtensorMap tk = make_tmap_bf16_3d(k, ks, p.Sk, p.B, ks, ks * p.Sk, 64, CQ::BK, 1);
    const CUtensorMap tv = make_tmap_bf16_3d(v, vs, p.Sk, p.B, vs, vs * p.Sk, 64, CQ::BK, 1);
    const int grid = p.B * p.H * ((p.Sq + CQ::BQ - 1) / CQ::BQ);
    kdq<<<grid, NUM_THREADS, CQ::SMEM, s>>>(tq, tdo, tk, tv, p);
    check_cuda(cudaGetLastError(), "attn_bwd_dq launch");
  }
}
}  // namespace attn_impl

void attn_fwd(const void* q, const void* k, const void* v, void* o, float* lse, int B, int Sq, int Sk, int H, int Hk,
              int Dqk, int Dv, bool causal, float scale, cudaStream_t s, const int* doc_start,
              const int* doc_end) {
  using namespace attn_impl;
  if (B == 0 || Sq == 0) return;
  if (doc_start != nullptr && (Sq != Sk || !causal || !((Dqk == 128 && Dv == 128) || (Dqk == 64 && Dv == 64))))
    throw std::runtime_error("attention: packed-document masks need causal self-attention with head dims 64 or 128");
  Params p;
  p.doc_start = doc_start;
  p.doc_end = doc_end;
  p.B = B;
  p.Sq = Sq;
  p.Sk = Sk;
  p.H = H;
  p.Hk = Hk;
  p.causal = causal ? 1 : 0;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.o = static_cast<__nv_bfloat16*>(o);
  p.lse = lse;
  p.num_qtiles = (Sq + BM - 1) / BM;
  if (Dqk == 128 && Dv == 128) launch_fwd2<128, 128>(q, k, v, p, s);
  else if (Dqk == 64 && Dv == 64) launch_fwd2<64, 64>(q, k, v, p, s);
  else if (Dqk == 192 && Dv == 128) launch_fwd<192, 128, 64>(q, k, v, p, Dqk, Dv, s);
  else throw std::runtime_error("attention: unsupported head dims (supported: 64/64, 128/128, 192/128)");
}

void attn_bwd(const void* dout, const void* q, const void* k, const void* v, const void* o, const float* lse,
              void* dq, void* dk, void* dv, float* dq_acc, float* delta, int B, int Sq, int Sk, int H, int Hk,
              int Dqk, int Dv, bool causal, float scale, cudaStream_t s, const float* dlse, const int* doc_start,
              const int* doc_end) {
  using namespace attn_impl;
  (void)dq_acc;
  if (doc_start != nullptr && (Sq != Sk || !causal))
    throw std::runtime_error("attention bwd: packed-document masks need causal self-attention");
  if (B == 0 || Sq == 0 || Sk == 0) return;
  const int64_t rows = (int64_t)B * Sq * H;
  attn_bwd_delta_kernel<<<static_cast<unsigned>((rows * 32 + 255) / 256), 256, 0, s>>>(
      static_cast<const __nv_bfloat16*>(dout), static_cast<const __nv_bfloat16*>(o), delta, dlse, B, Sq, H, Dv);
  check_cuda(cudaGetLastError(), "attn_bwd_delta");
  BwdParams p;
  p.B = B;
  p.Sq = Sq;
  p.Sk = Sk;
  p.H = H;
  p.Hk = Hk;
  p.causal = causal ? 1 : 0;
  p.scale = scale;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.lse = lse;
  p.delta = delta;
  p.dk = static_cast<__nv_bfloat16*>(dk);
  p.dv = static_cast<__nv_bfloat16*>(dv);
  p.dq = static_cast<__nv_bfloat16*>(dq);
  p.doc_start = doc_start;
  p.doc_end = doc_end;
  if (Dqk == 128 && Dv == 128) launch_bwd<128, 128, 2>(dout, q, k, v, p, s);
  else if (Dqk == 64 && Dv == 64) launch_bwd<64, 64, 2>(dout, q, k, v, p, s);
  else if (Dqk == 192 && Dv == 128) launch_bwd<192, 128, 1>(dout, q, k, v, p, s);
  else throw std::runtime_error("attention bwd: unsupported head dims (supported: 64/64, 128/128, 192/128)");
}

int attn_error_code(bool reset) {
  int v = 0;
  check_cuda(cudaMemcpyFromSymbol(&v, attn_impl::g_err, sizeof(int)), "attn error read");
  if (reset) {
    int z = 0;
    check_cuda(cudaMemcpyToSymbol(attn_impl::g_err, &z, sizeof(int)), "attn error reset");
  }
  return v;
}

}  // namespace ttb
