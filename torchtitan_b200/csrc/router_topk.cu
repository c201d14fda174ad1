// MoE token-choice routing selection in one launch: for every token, the expert scores
// (sigmoid or softmax of the router logits), the load-balancing bias added for the choice
// only, group-limited selection (keep the ``n_limited`` groups whose two best choices sum
// highest, DeepSeek-V3 style), the top-k experts, and the per-expert token counts.
//
// One warp per token; lane l holds experts l, l + 32, ... (E <= 32 * MAX_PER_LANE) in
// registers.  Top-k is k rounds of a warp arg-max (ties go to the lower expert index).
// The differentiable part of routing (gathering the scores of the chosen experts,
// normalising and scaling them) stays in PyTorch on the returned indices.
#include <cuda_runtime.h>

#include <stdexcept>

#include "launch_api.h"

namespace ttb {
namespace router_impl {

constexpr int MAX_PER_LANE = 16;  // E <= 512
constexpr int WARPS = 8;

__device__ __forceinline__ void warp_argmax(float& v, int& i) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, off);
    const int oi = __shfl_xor_sync(0xffffffffu, i, off);
    if (ov > v || (ov == v && oi < i)) {
      v = ov;
      i = oi;
    }
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}

__global__ void __launch_bounds__(WARPS * 32) router_kernel(const float* __restrict__ logits,
                                                            const float* __restrict__ bias, int64_t T, int E,
                                                            int top_k, int sigmoid, int n_groups, int n_limited,
                                                            int64_t* __restrict__ idx_out,
                                                            int32_t* __restrict__ counts) {
  const int lane = threadIdx.x % 32;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * WARPS + threadIdx.x / 32;
  if (t >= T) return;
  const float* row = logits + t * E;
  float s[MAX_PER_LANE];
  const float NEG = -INFINITY;
  float mx = NEG;
#pragma unroll
  for (int j = 0; j < MAX_PER_LANE; ++j) {
    const int e = lane + 32 * j;
    s[j] = e < E ? row[e] : NEG;
    mx = fmaxf(mx, s[j]);
  }
  if (sigmoid) {
#pragma unroll
    for (int j = 0; j < MAX_PER_LANE; ++j) s[j] = (lane + 32 * j) < E ? 1.f / (1.f + __expf(-s[j])) : NEG;
  } else {
    mx = warp_max(mx);
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < MAX_PER_LANE; ++j) {
      s[j] = (lane + 32 * j) < E ? __expf(s[j] - mx) : 0.f;
      sum += s[j];
    }
    sum = warp_sum(sum);
#pragma unroll
    for (int j = 0; j < MAX_PER_LANE; ++j) s[j] = (lane + 32 * j) < E ? s[j] / sum : NEG;
  }
  if (bias != nullptr) {
#pragma unroll
    for (int j = 0; j < MAX_PER_LANE; ++j)
      if (lane + 32 * j < E) s[j] += bias[lane + 32 * j];
  }
  if (n_groups > 1) {
    // group score = sum of the group's two best choices; keep the n_limited best groups
    const int per = E / n_groups;
    unsigned keep = 0;  // bit g set: group g kept (n_groups <= 32)
    float gscore_mine = NEG;  // lane g < n_groups holds group g's score
    for (int g = 0; g < n_groups; ++g) {
      float b1 = NEG, b2 = NEG;
#pragma unroll
      for (int j = 0; j < MAX_PER_LANE; ++j) {
        const int e = lane + 32 * j;
        if (e < E && e / per == g) {
          if (s[j] > b1) {
            b2 = b1;
            b1 = s[j];
          } else if (s[j] > b2) {
            b2 = s[j];
          }
        }
      }
      // warp-wide two best of the group
      float m1 = b1;
      int dummy = lane;
      warp_argmax(m1, dummy);
      float c2 = (b1 == m1 && lane == dummy) ? b2 : b1;  // the winner's lane offers its second best
      c2 = warp_max(c2);
      if (lane == g) gscore_mine = m1 + c2;
    }
    for (int r = 0; r < n_limited; ++r) {
      float v = lane < n_groups && !((keep >> lane) & 1u) ? gscore_mine : NEG;
      int i = lane;
      warp_argmax(v, i);
      keep |= 1u << i;
    }
#pragma unroll
    for (int j = 0; j < MAX_PER_LANE; ++j) {
      const int e = lane + 32 * j;
      if (e < E && !((keep >> (e / per)) & 1u)) s[j] = NEG;
    }
  }
  for (int r = 0; r < top_k; ++r) {
    float v = NEG;
    int i = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < MAX_PER_LANE; ++j) {
      const int e = lane + 32 * j;
      if (e < E && (s[j] > v || (s[j] == v && e < i))) {
        v = s[j];
        i = e;
      }
    }
    warp_argmax(v, i);
    if (lane == 0) {
      idx_out[t * top_k + r] = i;
      atomicAdd(counts + i, 1);
    }
#pragma unroll
    for (int j = 0; j < MAX_PER_LANE; ++j)  // remove the chosen expert
      if (lane + 32 * j == i) s[j] = NEG;
  }
}

}  // namespace router_impl

void router_topk(const float* logits, const float* bias, int64_t T, int E, int top_k, bool sigmoid, int n_groups,
                 int n_limited, int64_t* idx, int32_t* counts, cudaStream_t s) {
  using namespace router_impl;
  if (E > 32 * MAX_PER_LANE || E < 1) throw std::runtime_error("router_topk: 1 <= num_experts <= 512");
  if (top_k < 1 || top_k > E) throw std::runtime_error("router_topk: bad top_k");
  if (n_groups > 1 && (n_groups > 32 || E % n_groups || n_limited < 1 || n_limited > n_groups))
    throw std::runtime_error("router_topk: bad expert groups");
  check_cuda(cudaMemsetAsync(counts, 0, sizeof(int32_t) * E, s), "router counts clear");
  if (T == 0) return;
  const unsigned grid = static_cast<unsigned>((T + WARPS - 1) / WARPS);
  router_kernel<<<grid, WARPS * 32, 0, s>>>(logits, bias, T, E, top_k, sigmoid ? 1 : 0, n_groups, n_limited, idx,
                                            counts);
  check_cuda(cudaGetLastError(), "router_topk launch");
}

}  // namespace ttb
