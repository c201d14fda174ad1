// Chunk preparation of the chunked KDA forward, and its backward, as two memory-bound kernels
// (one thread per (sequence, head, chunk, feature column); rows walked in order, so the
// within-chunk cumulative sum is a running register):
//
//   inputs  q, k, g   [B, T, H, K] fp32 (q already scaled), rows past T read as 0
//   outputs (chunk layout [B*H, NT, C, K], or [B*H, NT, K] for decay)
//     qc = q, kc = k                       (chunked copies)
//     G  = cumsum_c g                      (within-chunk log decay)
//     kg = exp(G) * k,  qg = exp(G) * q
//     kd = exp(G_last - G) * k,  decay = exp(G_last)
//
// Backward (upstream gradients of the outputs, any may be absent; G saved from the forward):
//   dq = dqc + dqg * exp(G)
//   dk = dkc + dkg * exp(G) + dkd * exp(G_last - G)
//   dG = dG_in + dkg * kg + dqg * qg - dkd * kd,   dG_last += sum_c dkd * kd + ddecay * decay
//   dg = reverse cumsum_c dG
#include <cuda_runtime.h>

#include <stdexcept>

#include "launch_api.h"

namespace ttb {
namespace kprep {

constexpr int NT = 128;

struct Geo {
  int B, T, H, K, C, NT_;  // NT_: chunks per sequence
};

__device__ __forceinline__ size_t in_off(const Geo& g, int b, int t, int h, int d) {
  return ((static_cast<size_t>(b) * g.T + t) * g.H + h) * g.K + d;
}

// grid: (B*H*NT_ chunks, ceil(K / NT))
__global__ void __launch_bounds__(NT) prep_fwd_kernel(const float* __restrict__ q, const float* __restrict__ k,
                                                      const float* __restrict__ g, Geo geo, float* __restrict__ qc,
                                                      float* __restrict__ kc, float* __restrict__ G,
                                                      float* __restrict__ kg, float* __restrict__ qg,
                                                      float* __restrict__ kd, float* __restrict__ decay) {
  const int d = blockIdx.y * NT + threadIdx.x;
  if (d >= geo.K) return;
  const int chunk = blockIdx.x;  // (b*H + h)*NT_ + n
  const int n = chunk % geo.NT_, bh = chunk / geo.NT_;
  const int h = bh % geo.H, b = bh / geo.H;
  const size_t ob = static_cast<size_t>(chunk) * geo.C * geo.K + d;
  // pass 1: G and the chunk copies; keep the last G for pass 2
  float run = 0.f;
  for (int c = 0; c < geo.C; ++c) {
    const int t = n * geo.C + c;
    float vq = 0.f, vk = 0.f, vg = 0.f;
    if (t < geo.T) {
      const size_t o = in_off(geo, b, t, h, d);
      vq = q[o];
      vk = k[o];
      vg = g[o];
    }
    run += vg;
    const size_t oc = ob + static_cast<size_t>(c) * geo.K;
    qc[oc] = vq;
    kc[oc] = vk;
    G[oc] = run;
    const float e = __expf(run);
    kg[oc] = e * vk;
    qg[oc] = e * vq;
  }
  const float last = run;
  decay[static_cast<size_t>(chunk) * geo.K + d] = __expf(last);
  for (int c = 0; c < geo.C; ++c) {
    const size_t oc = ob + static_cast<size_t>(c) * geo.K;
    kd[oc] = __expf(last - G[oc]) * kc[oc];
  }
}

__global__ void __launch_bounds__(NT) prep_bwd_kernel(const float* __restrict__ q, const float* __restrict__ k,
                                                      const float* __restrict__ G, Geo geo,
                                                      const float* __restrict__ dqc, const float* __restrict__ dkc,
                                                      const float* __restrict__ dG, const float* __restrict__ dkg,
                                                      const float* __restrict__ dqg, const float* __restrict__ dkd,
                                                      const float* __restrict__ ddecay, float* __restrict__ dq,
                                                      float* __restrict__ dk, float* __restrict__ dg) {
  const int d = blockIdx.y * NT + threadIdx.x;
  if (d >= geo.K) return;
  const int chunk = blockIdx.x;
  const int n = chunk % geo.NT_, bh = chunk / geo.NT_;
  const int h = bh % geo.H, b = bh / geo.H;
  const size_t ob = static_cast<size_t>(chunk) * geo.C * geo.K + d;
  const float last = G[ob + static_cast<size_t>(geo.C - 1) * geo.K];
  // the last row's extra gradient collects every kd term and the decay term
  float dlast = ddecay ? ddecay[static_cast<size_t>(chunk) * geo.K + d] * __expf(last) : 0.f;
  for (int c = 0; c < geo.C; ++c) {
    const int t = n * geo.C + c;
    if (t >= geo.T) break;
    const size_t oc = ob + static_cast<size_t>(c) * geo.K;
    const float vk = k[in_off(geo, b, t, h, d)];
    dlast += (dkd ? dkd[oc] : 0.f) * __expf(last - G[oc]) * vk;
  }
  // reverse walk: dg[c] = sum_{c' >= c} dG_total[c']
  float acc = 0.f;
  for (int c = geo.C - 1; c >= 0; --c) {
    const int t = n * geo.C + c;
    const size_t oc = ob + static_cast<size_t>(c) * geo.K;
    const float Gc = G[oc];
    const float e = __expf(Gc), ed = __expf(last - Gc);
    float vq = 0.f, vk = 0.f;
    size_t o = 0;
    if (t < geo.T) {
      o = in_off(geo, b, t, h, d);
      vq = q[o];
      vk = k[o];
    }
    const float gkg = dkg ? dkg[oc] : 0.f, gqg = dqg ? dqg[oc] : 0.f, gkd = dkd ? dkd[oc] : 0.f;
    float dGc = (dG ? dG[oc] : 0.f) + gkg * e * vk + gqg * e * vq - gkd * ed * vk;
    if (c == geo.C - 1) dGc += dlast;
    acc += dGc;
    if (t < geo.T) {
      dq[o] = (dqc ? dqc[oc] : 0.f) + gqg * e;
      dk[o] = (dkc ? dkc[oc] : 0.f) + gkg * e + gkd * ed;
      dg[o] = acc;
    }
  }
}

}  // namespace kprep

void kda_prep_fwd(const float* q, const float* k, const float* g, int B, int T, int H, int K, int C, float* qc,
                  float* kc, float* G, float* kg, float* qg, float* kd, float* decay, cudaStream_t s) {
  using namespace kprep;
  const int nt = (T + C - 1) / C;
  if (B == 0 || nt == 0) return;
  const Geo geo{B, T, H, K, C, nt};
  const dim3 grid(static_cast<unsigned>(B * H * nt), (K + NT - 1) / NT);
  prep_fwd_kernel<<<grid, NT, 0, s>>>(q, k, g, geo, qc, kc, G, kg, qg, kd, decay);
  check_cuda(cudaGetLastError(), "kda_prep_fwd");
}

void kda_prep_bwd(const float* q, const float* k, const float* G, int B, int T, int H, int K, int C,
                  const float* dqc, const float* dkc, const float* dG, const float* dkg, const float* dqg,
                  const float* dkd, const float* ddecay, float* dq, float* dk, float* dg, cudaStream_t s) {
  using namespace kprep;
  const int nt = (T + C - 1) / C;
  if (B == 0 || nt == 0) return;
  const Geo geo{B, T, H, K, C, nt};
  const dim3 grid(static_cast<unsigned>(B * H * nt), (K + NT - 1) / NT);
  prep_bwd_kernel<<<grid, NT, 0, s>>>(q, k, G, geo, dqc, dkc, dG, dkg, dqg, dkd, ddecay, dq, dk, dg);
  check_cuda(cudaGetLastError(), "kda_prep_bwd");
}

}  // namespace ttb
