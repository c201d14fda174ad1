// Expert-parallel row movement over NVLink peer memory (no NCCL).
//
// * ep_scatter_rows: row i of `src` is stored into rank dest_rank[i]'s buffer at
//   row dest_row[i] (P2P stores of 16-byte vectors).  Used to place routed tokens
//   directly into each expert owner's padded expert-major layout (dispatch), and
//   output gradients back into that layout (combine backward).
// * ep_gather_rows: row i of `dst` is loaded from rank src_rank[i]'s buffer at
//   row src_row[i] (P2P loads).  Used to fetch expert outputs back into token
//   order (combine), and input gradients (dispatch backward).
// One warp moves one row; D * 2 bytes must be a multiple of 16.  Ordering with
// respect to the peers is established by the caller's epoch barriers
// (dp_barrier), which bracket every call.  Every peer row index is checked against the
// destination buffer's capacity; an out-of-range index is skipped and recorded (ep_error_code).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "launch_api.h"

namespace ttb {
namespace ep_impl {

constexpr int kMaxPeers = 8;

// first out-of-capacity row index seen (a count or plan mismatch between ranks): the row is
// skipped rather than written past the end of a peer's buffer; the host reads it between steps
__device__ int g_ep_err;

__device__ __forceinline__ bool row_ok(int64_t row, int64_t cap) {
  if (row >= 0 && row < cap) return true;
  atomicCAS(&g_ep_err, 0, 1);
  return false;
}

struct PeerBases {
  __nv_bfloat16* p[kMaxPeers];
};

__global__ void __launch_bounds__(256) scatter_rows_kernel(const __nv_bfloat16* __restrict__ src, int64_t n,
                                                           int row_vecs, const int32_t* __restrict__ dest_rank,
                                                           const int64_t* __restrict__ dest_row,
                                                           const __grid_constant__ PeerBases peers, int world,
                                                           int64_t cap_rows) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t i = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); i < n; i += warps) {
    const int r = dest_rank[i];
    if (r < 0 || r >= world) continue;  // dropped row
    if (!row_ok(dest_row[i], cap_rows)) continue;
    const uint4* s = reinterpret_cast<const uint4*>(src + i * (int64_t)row_vecs * 8);
    uint4* d = reinterpret_cast<uint4*>(peers.p[r] + dest_row[i] * (int64_t)row_vecs * 8);
    for (int v = lane; v < row_vecs; v += 32) d[v] = s[v];
  }
}

__global__ void __launch_bounds__(256) gather_rows_kernel(__nv_bfloat16* __restrict__ dst, int64_t n,
                                                          int row_vecs, const int32_t* __restrict__ src_rank,
                                                          const int64_t* __restrict__ src_row,
                                                          const __grid_constant__ PeerBases peers, int world,
                                                          int64_t cap_rows) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t i = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); i < n; i += warps) {
    const int r = src_rank[i];
    uint4* d = reinterpret_cast<uint4*>(dst + i * (int64_t)row_vecs * 8);
    if (r < 0 || r >= world || !row_ok(src_row[i], cap_rows)) {
      for (int v = lane; v < row_vecs; v += 32) d[v] = make_uint4(0, 0, 0, 0);
      continue;
    }
    const uint4* s = reinterpret_cast<const uint4*>(peers.p[r] + src_row[i] * (int64_t)row_vecs * 8);
    for (int v = lane; v < row_vecs; v += 32) d[v] = s[v];
  }
}

PeerBases make_bases(void* const* bases, int world) {
  if (world < 1 || world > kMaxPeers) throw std::runtime_error("ep: world size must be 1..8");
  PeerBases b;
  for (int j = 0; j < kMaxPeers; ++j) b.p[j] = j < world ? static_cast<__nv_bfloat16*>(bases[j]) : nullptr;
  return b;
}

int grid_for(int64_t n) {
  const int64_t blocks = (n + 7) / 8;  // 8 warps per block, one row per warp
  return static_cast<int>(blocks < 1184 ? (blocks < 1 ? 1 : blocks) : 1184);  // 148 SMs x 8
}

}  // namespace ep_impl

void ep_scatter_rows(const void* src, int64_t n, int d, const int32_t* dest_rank, const int64_t* dest_row,
                     void* const* peer_bases, int world, int64_t cap_rows, cudaStream_t s) {
  using namespace ep_impl;
  if (d % 8) throw std::runtime_error("ep_scatter_rows: row length must be a multiple of 8 bf16");
  if (n == 0) return;
  scatter_rows_kernel<<<grid_for(n), 256, 0, s>>>(static_cast<const __nv_bfloat16*>(src), n, d / 8, dest_rank,
                                                   dest_row, make_bases(peer_bases, world), world, cap_rows);
  check_cuda(cudaGetLastError(), "ep scatter launch");
}

void ep_gather_rows(void* dst, int64_t n, int d, const int32_t* src_rank, const int64_t* src_row,
                    void* const* peer_bases, int world, int64_t cap_rows, cudaStream_t s) {
  using namespace ep_impl;
  if (d % 8) throw std::runtime_error("ep_gather_rows: row length must be a multiple of 8 bf16");
  if (n == 0) return;
  gather_rows_kernel<<<grid_for(n), 256, 0, s>>>(static_cast<__nv_bfloat16*>(dst), n, d / 8, src_rank, src_row,
                                                  make_bases(peer_bases, world), world, cap_rows);
  check_cuda(cudaGetLastError(), "ep gather launch");
}

int ep_error_code(bool reset) {
  int v = 0;
  check_cuda(cudaMemcpyFromSymbol(&v, ep_impl::g_ep_err, sizeof(int)), "ep error read");
  if (reset && v) {
    int z = 0;
    check_cuda(cudaMemcpyToSymbol(ep_impl::g_ep_err, &z, sizeof(int)), "ep error reset");
  }
  return v;
}

}  // namespace ttb
