// Inter-chunk recurrence of chunked KDA (Kimi Delta Attention), forward and
// backward, as one launch each instead of a host loop of small matmuls per chunk.
//
// Per head (state S in R^{K x V}, chunks n = 0..NT-1, chunk length C):
//   v'_n    = u_n - w_n S_n                          [C, V]
//   o_n     = qg_n S_n + Aqk_n v'_n                   [C, V]
//   S_{n+1} = diag(d_n) S_n + kdec_n^T v'_n           [K, V]      (S_0 = 0)
// Every column of S evolves on its own, so the grid is (V slices, heads): each CTA
// owns VS columns of one head's state in shared memory and walks the chunks in order.
// The forward stores each chunk's starting state (for the backward).
//
// Backward (reverse walk, dS carried in shared memory, dS_NT = 0):
//   dv'   = Aqk^T dO + kdec dS_{n+1}
//   du    = dv'
//   dS_n  = qg^T dO + diag(d) dS_{n+1} - w^T dv'
// and, summed over this CTA's columns (the host adds the V slices):
//   dqg = dO S_n^T,  dw = -dv' S_n^T,  dkdec = v' dS_{n+1}^T,  dAqk = dO v'^T,
//   dd[k] = sum_v dS_{n+1}[k, v] S_n[k, v].
// fp32 throughout (the state recurrence is precision-sensitive); rows of the
// shared-memory tiles are padded by one word so column walks are bank-conflict free.
#include <cuda_runtime.h>

#include <stdexcept>

#include "launch_api.h"

namespace ttb {
namespace kscan {

constexpr int NT_THREADS = 256;

struct Dims {
  int NT, C, K, V, VS;
};

__device__ __forceinline__ void load_rows(float* dst, int ld_dst, const float* src, int rows, int cols,
                                          int ld_src) {
  for (int x = threadIdx.x; x < rows * cols; x += NT_THREADS) {
    const int r = x / cols, c = x - r * cols;
    dst[r * ld_dst + c] = src[static_cast<size_t>(r) * ld_src + c];
  }
}

__global__ void __launch_bounds__(NT_THREADS, 1) scan_fwd_kernel(const float* __restrict__ u, const float* __restrict__ w,
                                                              const float* __restrict__ qg,
                                                              const float* __restrict__ Aqk,
                                                              const float* __restrict__ kdec,
                                                              const float* __restrict__ dec, float* __restrict__ o,
                                                              float* __restrict__ states, float* __restrict__ final_S,
                                                              Dims d) {
  extern __shared__ float sm[];
  const int C = d.C, K = d.K, V = d.V, VS = d.VS;
  const int PK = K + 1, PC = C + 1, PV = VS + 1;
  float* S = sm;                // [K][PV]
  float* sw = S + K * PV;       // [C][PK]
  float* sq = sw + C * PK;      // [C][PK]
  float* skd = sq + C * PK;     // [C][PK]
  float* sA = skd + C * PK;     // [C][PC]
  float* sv = sA + C * PC;      // [C][PV]  u, then v'
  float* sd = sv + C * PV;      // [K]
  const int v0 = blockIdx.x * VS;
  const size_t bh = blockIdx.y;
  for (int x = threadIdx.x; x < K * PV; x += NT_THREADS) S[x] = 0.f;
  __syncthreads();
  for (int n = 0; n < d.NT; ++n) {
    const size_t ck = (bh * d.NT + n) * static_cast<size_t>(C);
    load_rows(sw, PK, w + ck * K, C, K, K);
    load_rows(sq, PK, qg + ck * K, C, K, K);
    load_rows(skd, PK, kdec + ck * K, C, K, K);
    load_rows(sA, PC, Aqk + ck * C, C, C, C);
    load_rows(sv, PV, u + ck * V + v0, C, VS, V);
    for (int k = threadIdx.x; k < K; k += NT_THREADS) sd[k] = dec[(bh * d.NT + n) * K + k];
    // chunk-start state for the backward
    float* st = states + ((bh * d.NT + n) * static_cast<size_t>(K)) * V + v0;
    for (int x = threadIdx.x; x < K * VS; x += NT_THREADS) {
      const int k = x / VS, j = x - k * VS;
      st[static_cast<size_t>(k) * V + j] = S[k * PV + j];
    }
    __syncthreads();
    // v' = u - w S
    for (int x = threadIdx.x; x < C * VS; x += NT_THREADS) {
      const int i = x / VS, j = x - i * VS;
      float acc = sv[i * PV + j];
      const float* wi = sw + i * PK;
#pragma unroll 8
      for (int k = 0; k < K; ++k) acc -= wi[k] * S[k * PV + j];
      sv[i * PV + j] = acc;
    }
    __syncthreads();
    // o = qg S + Aqk v'
    float* on = o + ck * V + v0;
    for (int x = threadIdx.x; x < C * VS; x += NT_THREADS) {
      const int i = x / VS, j = x - i * VS;
      float acc = 0.f;
      const float* qi = sq + i * PK;
#pragma unroll 8
      for (int k = 0; k < K; ++k) acc += qi[k] * S[k * PV + j];
      const float* ai = sA + i * PC;
#pragma unroll 8
      for (int c = 0; c < C; ++c) acc += ai[c] * sv[c * PV + j];
      on[static_cast<size_t>(i) * V + j] = acc;
    }
    __syncthreads();
    // S <- diag(d) S + kdec^T v'   (each element read and written by one thread)
    for (int x = threadIdx.x; x < K * VS; x += NT_THREADS) {
      const int k = x / VS, j = x - k * VS;
      float acc = sd[k] * S[k * PV + j];
#pragma unroll 8
      for (int c = 0; c < C; ++c) acc += skd[c * PK + k] * sv[c * PV + j];
      S[k * PV + j] = acc;
    }
    __syncthreads();
  }
  if (final_S != nullptr) {
    float* fs = final_S + bh * static_cast<size_t>(K) * V + v0;
    for (int x = threadIdx.x; x < K * VS; x += NT_THREADS) {
      const int k = x / VS, j = x - k * VS;
      fs[static_cast<size_t>(k) * V + j] = S[k * PV + j];
    }
  }
}

__global__ void __launch_bounds__(NT_THREADS, 1) scan_bwd_kernel(
    const float* __restrict__ dO, const float* __restrict__ u, const float* __restrict__ w,
    const float* __restrict__ qg, const float* __restrict__ Aqk, const float* __restrict__ kdec,
    const float* __restrict__ dec, const float* __restrict__ states, float* __restrict__ du,
    float* __restrict__ p_dqg, float* __restrict__ p_dw, float* __restrict__ p_dkdec, float* __restrict__ p_dA,
    float* __restrict__ p_dd, Dims d, int64_t slice_stride_ck, int64_t slice_stride_cc, int64_t slice_stride_k) {
  extern __shared__ float sm[];
  const int C = d.C, K = d.K, V = d.V, VS = d.VS;
  const int PK = K + 1, PC = C + 1, PV = VS + 1;
  float* S = sm;                // [K][PV] chunk-start state
  float* dS = S + K * PV;       // [K][PV] carried dS_{n+1}
  float* sw = dS + K * PV;      // [C][PK]
  float* sq = sw + C * PK;      // [C][PK]
  float* skd = sq + C * PK;     // [C][PK]
  float* sA = skd + C * PK;     // [C][PC]
  float* sdo = sA + C * PC;     // [C][PV]
  float* sv = sdo + C * PV;     // [C][PV] v'
  float* sdv = sv + C * PV;     // [C][PV] dv'
  float* sd = sdv + C * PV;     // [K]
  const int slice = blockIdx.x;
  const int v0 = slice * VS;
  const size_t bh = blockIdx.y;
  for (int x = threadIdx.x; x < K * PV; x += NT_THREADS) dS[x] = 0.f;
  __syncthreads();
  for (int n = d.NT - 1; n >= 0; --n) {
    const size_t cn = bh * d.NT + n;
    const size_t ck = cn * static_cast<size_t>(C);
    load_rows(sw, PK, w + ck * K, C, K, K);
    load_rows(sq, PK, qg + ck * K, C, K, K);
    load_rows(skd, PK, kdec + ck * K, C, K, K);
    load_rows(sA, PC, Aqk + ck * C, C, C, C);
    load_rows(sdo, PV, dO + ck * V + v0, C, VS, V);
    load_rows(sv, PV, u + ck * V + v0, C, VS, V);
    load_rows(S, PV, states + cn * static_cast<size_t>(K) * V + v0, K, VS, V);
    for (int k = threadIdx.x; k < K; k += NT_THREADS) sd[k] = dec[cn * K + k];
    __syncthreads();
    // v' = u - w S ;  dv' = Aqk^T dO + kdec dS
    for (int x = threadIdx.x; x < C * VS; x += NT_THREADS) {
      const int i = x / VS, j = x - i * VS;
      float acc = sv[i * PV + j], dacc = 0.f;
      const float* wi = sw + i * PK;
      const float* ki = skd + i * PK;
#pragma unroll 8
      for (int k = 0; k < K; ++k) {
        acc -= wi[k] * S[k * PV + j];
        dacc += ki[k] * dS[k * PV + j];
      }
#pragma unroll 8
      for (int c = 0; c < C; ++c) dacc += sA[c * PC + i] * sdo[c * PV + j];
      sv[i * PV + j] = acc;
      sdv[i * PV + j] = dacc;
      du[ck * V + static_cast<size_t>(i) * V + v0 + j] = dacc;
    }
    __syncthreads();
    // per-slice partial sums over this CTA's columns
    const size_t pck = slice * slice_stride_ck + ck * K;  // [C][K] block of chunk n
    for (int x = threadIdx.x; x < C * K; x += NT_THREADS) {
      const int i = x / K, k = x - i * K;
      float aq = 0.f, aw = 0.f, ak = 0.f;
#pragma unroll 8
      for (int j = 0; j < VS; ++j) {
        const float s = S[k * PV + j];
        aq += sdo[i * PV + j] * s;
        aw -= sdv[i * PV + j] * s;
        ak += sv[i * PV + j] * dS[k * PV + j];
      }
      p_dqg[pck + x] = aq;
      p_dw[pck + x] = aw;
      p_dkdec[pck + x] = ak;
    }
    const size_t pcc = slice * slice_stride_cc + ck * C;
    for (int x = threadIdx.x; x < C * C; x += NT_THREADS) {
      const int i = x / C, c = x - i * C;
      float a = 0.f;
#pragma unroll 8
      for (int j = 0; j < VS; ++j) a += sdo[i * PV + j] * sv[c * PV + j];
      p_dA[pcc + x] = a;
    }
    for (int k = threadIdx.x; k < K; k += NT_THREADS) {
      float a = 0.f;
      for (int j = 0; j < VS; ++j) a += dS[k * PV + j] * S[k * PV + j];
      p_dd[slice * slice_stride_k + cn * K + k] = a;
    }
    __syncthreads();
    // dS_n = qg^T dO + diag(d) dS_{n+1} - w^T dv'
    for (int x = threadIdx.x; x < K * VS; x += NT_THREADS) {
      const int k = x / VS, j = x - k * VS;
      float acc = sd[k] * dS[k * PV + j];
#pragma unroll 8
      for (int i = 0; i < C; ++i) acc += sq[i * PK + k] * sdo[i * PV + j] - sw[i * PK + k] * sdv[i * PV + j];
      dS[k * PV + j] = acc;
    }
    __syncthreads();
  }
}

size_t fwd_smem(int C, int K, int VS) {
  return sizeof(float) * (static_cast<size_t>(K) * (VS + 1) + 3 * static_cast<size_t>(C) * (K + 1) +
                          static_cast<size_t>(C) * (C + 1) + static_cast<size_t>(C) * (VS + 1) + K);
}
size_t bwd_smem(int C, int K, int VS) {
  return sizeof(float) * (2 * static_cast<size_t>(K) * (VS + 1) + 3 * static_cast<size_t>(C) * (K + 1) +
                          static_cast<size_t>(C) * (C + 1) + 3 * static_cast<size_t>(C) * (VS + 1) + K);
}

void check_dims(int C, int K, int V, int VS, size_t smem) {
  if (C <= 0 || K <= 0 || V <= 0 || VS <= 0 || V % VS) throw std::runtime_error("kda_scan: bad dimensions");
  if (smem > 227 * 1024) throw std::runtime_error("kda_scan: chunk x head dims too large for shared memory");
}

}  // namespace kscan

void kda_scan_fwd(const float* u, const float* w, const float* qg, const float* Aqk, const float* kdec,
                  const float* dec, float* o, float* states, float* final_S, int64_t BH, int NT, int C, int K, int V,
                  int VS, cudaStream_t s) {
  using namespace kscan;
  if (BH == 0 || NT == 0) return;
  const size_t sm = fwd_smem(C, K, VS);
  check_dims(C, K, V, VS, sm);
  check_cuda(cudaFuncSetAttribute(scan_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm),
             "kda scan smem");
  const dim3 grid(V / VS, (unsigned)BH);
  scan_fwd_kernel<<<grid, NT_THREADS, sm, s>>>(u, w, qg, Aqk, kdec, dec, o, states, final_S, Dims{NT, C, K, V, VS});
  check_cuda(cudaGetLastError(), "kda scan fwd launch");
}

void kda_scan_bwd(const float* dO, const float* u, const float* w, const float* qg, const float* Aqk,
                  const float* kdec, const float* dec, const float* states, float* du, float* p_dqg, float* p_dw,
                  float* p_dkdec, float* p_dA, float* p_dd, int64_t BH, int NT, int C, int K, int V, int VS,
                  cudaStream_t s) {
  using namespace kscan;
  if (BH == 0 || NT == 0) return;
  const size_t sm = bwd_smem(C, K, VS);
  check_dims(C, K, V, VS, sm);
  check_cuda(cudaFuncSetAttribute(scan_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm),
             "kda scan smem");
  const dim3 grid(V / VS, (unsigned)BH);
  const int64_t sck = BH * NT * static_cast<int64_t>(C) * K, scc = BH * NT * static_cast<int64_t>(C) * C,
                sk = BH * NT * static_cast<int64_t>(K);
  scan_bwd_kernel<<<grid, NT_THREADS, sm, s>>>(dO, u, w, qg, Aqk, kdec, dec, states, du, p_dqg, p_dw, p_dkdec, p_dA,
                                               p_dd, Dims{NT, C, K, V, VS}, sck, scc, sk);
  check_cuda(cudaGetLastError(), "kda scan bwd launch");
}

}  // namespace ttb
