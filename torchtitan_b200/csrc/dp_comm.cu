// Data-parallel collectives over NVLink peer memory (symmetric buffers), no NCCL.
//
// * rs_bucket: reduce-scatter of one gradient bucket.  Rank r owns the r-th
//   1/W slice of the bucket; it signals every peer that its own bf16 gradient
//   bucket is complete (system-scope release), waits (bounded) until every peer
//   has signalled the same, then sums slice r of all W peers' buffers with
//   plain 16-byte P2P loads, accumulating in fp32 and writing the scaled fp32
//   shard gradient.  The transfer is the arithmetic: no staging buffer, no
//   separate cast/scale pass.
// * dp_barrier: epoch barrier across the W ranks through the same flags (used
//   after the optimizer's P2P stores of updated weights).
// Flags are uint32 epochs in each rank's signal pad; every wait gives up after
// ~20 s, records an error code readable by dp_error_code() and returns.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "launch_api.h"

namespace ttb {
namespace dp_impl {

__device__ int g_err;
__device__ int g_err_info[4];  // slot, epoch awaited, source rank, value seen (first failure)
// optional host-mapped (pinned) int[8]: [code, slot, epoch, source, value, ...] written on the first
// failure so a host thread sees it without any CUDA call while the stream is still busy
__device__ int* g_host_sink;
// generous: ranks may drift apart by a data-loader hiccup, a checkpoint write or a slow first step
constexpr uint64_t kDefaultLimitNs = 20000000000ull;
constexpr int kMaxWorld = 8;

struct PeerTable {
  const __nv_bfloat16* g[kMaxWorld];  // each rank's flat gradient buffer
  uint32_t* sig[kMaxWorld];           // each rank's signal pad (uint32 slots)
  int world, rank;
  uint64_t limit_ns;  // give up a wait after this long
};

__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint4 ld_cg_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

// slot layout in each signal pad: [slot_base + bucket * W + src_rank]
__device__ bool signal_and_wait(const PeerTable& t, int slot, uint32_t epoch, int code) {
  const uint64_t limit = t.limit_ns;
  __shared__ int ok;
  if (threadIdx.x == 0) ok = 1;
  __syncthreads();
  if (blockIdx.x == 0 && threadIdx.x < t.world) {
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    st_release_sys(t.sig[threadIdx.x] + slot * t.world + t.rank, epoch);
  }
  // once any wait of this process gave up, later waits return at once: a failed step
  // surfaces after one time limit instead of one limit per queued kernel
  if (threadIdx.x == 0 && *static_cast<volatile int*>(&g_err) != 0) ok = 0;
  __syncthreads();
  if (threadIdx.x == 0 && ok) {
    const uint32_t* mine = t.sig[t.rank] + slot * t.world;
    const uint64_t t0 = now_ns();
    for (int j = 0; j < t.world; ++j) {
      while (static_cast<int32_t>(ld_acquire_sys(mine + j) - epoch) < 0) {
        if (now_ns() - t0 > limit) {
          if (atomicCAS(&g_err, 0, code) == 0) {
            g_err_info[0] = slot;
            g_err_info[1] = static_cast<int>(epoch);
            g_err_info[2] = j;
            g_err_info[3] = static_cast<int>(ld_acquire_sys(mine + j));
            if (g_host_sink != nullptr) {
              volatile int* h = g_host_sink;
              h[1] = slot;
              h[2] = static_cast<int>(epoch);
              h[3] = j;
              h[4] = g_err_info[3];
              __threadfence_system();
              h[0] = code;
              __threadfence_system();
            }
          }
          ok = 0;
          j = t.world;
          break;
        }
      }
    }
  }
  __syncthreads();
  return ok != 0;
}

__global__ void __launch_bounds__(256) rs_bucket_kernel(PeerTable t, int64_t bucket_off, int64_t shard_len,
                                                         float* __restrict__ out, float scale, int slot,
                                                         uint32_t epoch) {
  if (!signal_and_wait(t, slot, epoch, 71)) return;
  const int64_t base = bucket_off + static_cast<int64_t>(t.rank) * shard_len;
  const int64_t n8 = shard_len / 8;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    uint4 v[kMaxWorld];
    // issue every peer's 16-byte load before consuming any: W requests in flight per thread
#pragma unroll
    for (int j = 0; j < kMaxWorld; ++j) {
      const int src = (t.rank + j) % t.world;  // stagger sources across ranks
      if (j < t.world) v[j] = ld_cg_v4(t.g[src] + base + i * 8);
    }
#pragma unroll
    for (int j = 0; j < kMaxWorld; ++j) {
      if (j >= t.world) break;
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v[j]);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float2 f = __bfloat1622float2(h[u]);
        acc[2 * u] += f.x;
        acc[2 * u + 1] += f.y;
      }
    }
    float4* o = reinterpret_cast<float4*>(out + i * 8);
    o[0] = make_float4(acc[0] * scale, acc[1] * scale, acc[2] * scale, acc[3] * scale);
    o[1] = make_float4(acc[4] * scale, acc[5] * scale, acc[6] * scale, acc[7] * scale);
  }
}

__global__ void dp_barrier_kernel(PeerTable t, int slot, uint32_t epoch) { signal_and_wait(t, slot, epoch, 72); }

PeerTable make_table(const void* const* grads, uint32_t* const* sigs, int world, int rank, double limit_s) {
  if (world < 1 || world > kMaxWorld) throw std::runtime_error("dp: world size must be 1..8");
  PeerTable t;
  for (int j = 0; j < kMaxWorld; ++j) {
    t.g[j] = j < world && grads ? static_cast<const __nv_bfloat16*>(grads[j]) : nullptr;
    t.sig[j] = j < world ? sigs[j] : nullptr;
  }
  t.world = world;
  t.rank = rank;
  t.limit_ns = limit_s > 0 ? static_cast<uint64_t>(limit_s * 1e9) : kDefaultLimitNs;
  return t;
}

}  // namespace dp_impl

void dp_reduce_scatter_bucket(const void* const* peer_grads, uint32_t* const* peer_sigs, int world, int rank,
                              int64_t bucket_off, int64_t bucket_len, float* out_shard, float scale, int slot,
                              uint32_t epoch, int num_ctas, cudaStream_t s, double limit_s) {
  using namespace dp_impl;
  if (bucket_len % (8 * world)) throw std::runtime_error("dp: bucket length must be a multiple of 8 * world");
  const PeerTable t = make_table(peer_grads, peer_sigs, world, rank, limit_s);
  rs_bucket_kernel<<<num_ctas, 256, 0, s>>>(t, bucket_off, bucket_len / world, out_shard, scale, slot, epoch);
  check_cuda(cudaGetLastError(), "dp rs launch");
}

void dp_barrier(uint32_t* const* peer_sigs, int world, int rank, int slot, uint32_t epoch, cudaStream_t s,
                double limit_s) {
  using namespace dp_impl;
  const PeerTable t = make_table(nullptr, peer_sigs, world, rank, limit_s);
  dp_barrier_kernel<<<1, 32, 0, s>>>(t, slot, epoch);
  check_cuda(cudaGetLastError(), "dp barrier launch");
}

void dp_set_error_sink(void* host_mapped_int8) {
  int* p = static_cast<int*>(host_mapped_int8);
  check_cuda(cudaMemcpyToSymbol(dp_impl::g_host_sink, &p, sizeof(int*)), "dp error sink");
}

void dp_error_info(int* out4) {
  check_cuda(cudaMemcpyFromSymbol(out4, dp_impl::g_err_info, 4 * sizeof(int)), "dp error info read");
}

int dp_error_code(bool reset) {
  int v = 0;
  check_cuda(cudaMemcpyFromSymbol(&v, dp_impl::g_err, sizeof(int)), "dp error read");
  if (reset) {
    int z = 0;
    check_cuda(cudaMemcpyToSymbol(dp_impl::g_err, &z, sizeof(int)), "dp error reset");
  }
  return v;
}

}  // namespace ttb
