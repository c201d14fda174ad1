// Multi-tensor AdamW (decoupled weight decay) for sm_100a.
//
// The host flattens every (param, grad, exp_avg, exp_avg_sq) quadruple into
// fixed-size chunks; one launch processes all chunks of all tensors.  Params
// are fp32 (master) or bf16, grads fp32 or bf16, moments fp32.  The chunk
// table travels as a kernel argument in batches, so nothing is allocated on
// the device.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <functional>
#include <vector>

#include "launch_api.h"

namespace ttb {
namespace {

constexpr int CHUNK = 65536;
constexpr int MAX_CHUNKS = 560;  // per launch: 560 x 56 B (+ peer table) fits the 32 KB kernel-parameter budget
constexpr int NT = 512;

struct Chunk {
  void* p;
  const void* g;
  float* m;
  float* v;
  int n;
  int8_t p_bf16;
  int8_t g_bf16;
  int8_t vec4;  // every pointer 16-byte aligned and n % 4 == 0: float4 path
  __nv_bfloat16* p_copy;  // optional bf16 copy written with the updated fp32 param
  int64_t peer_off;       // >= 0: also write the bf16 copy at this element offset of every peer buffer
};

// bf16 weight buffers of all data-parallel ranks (NVLink peer mappings, own rank included)
struct Peers {
  __nv_bfloat16* base[8];
  int n;
};

struct Table {
  Chunk c[MAX_CHUNKS];
};

__device__ __forceinline__ float ldv(const void* base, int64_t i, int8_t is_bf16) {
  return is_bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(base)[i]) : static_cast<const float*>(base)[i];
}

__device__ __forceinline__ float adam_update(float& pv, float g, float& m, float& v, float b1, float b2, float eps,
                                             float decay, float step_size, float bc2_sqrt) {
  m = b1 * m + (1.f - b1) * g;
  v = b2 * v + (1.f - b2) * g * g;
  pv = pv * decay - step_size * m / (sqrtf(v) / bc2_sqrt + eps);
  return pv;
}

// clip_total (optional): device sum of squared grad norms; grads are scaled by
// min(1, clip_max / (sqrt(total) + 1e-6)) on the fly (clipping fused into the step)
__device__ __forceinline__ void adamw_chunk(const Chunk& c, float lr, float b1, float b2, float eps, float wd,
                                            float bc1, float bc2_sqrt, const float* __restrict__ clip_total,
                                            float clip_max, const Peers& peers) {
  const float gs = clip_total ? fminf(clip_max / (sqrtf(*clip_total) + 1e-6f), 1.f) : 1.f;
  const float step_size = lr / bc1;
  const float decay = 1.f - lr * wd;
  if (c.vec4 && !c.p_bf16) {
    // fp32 master, bf16 or fp32 grad (and optionally bf16 compute copies): vector loads and stores
    float4* p4 = static_cast<float4*>(c.p);
    float4* m4 = reinterpret_cast<float4*>(c.m);
    float4* v4 = reinterpret_cast<float4*>(c.v);
    uint2* c4 = reinterpret_cast<uint2*>(c.p_copy);
    const bool copy = c4 != nullptr || c.peer_off >= 0;
    const int n4 = c.n / 4;
#pragma unroll 2
    for (int i = threadIdx.x; i < n4; i += NT) {
      float4 p = p4[i], m = m4[i], v = v4[i];
      float4 g;
      if (c.g_bf16) {
        const uint2 gr = static_cast<const uint2*>(c.g)[i];
        const float2 g01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&gr.x));
        const float2 g23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&gr.y));
        g = make_float4(g01.x, g01.y, g23.x, g23.y);
      } else {
        g = static_cast<const float4*>(c.g)[i];
      }
      g.x *= gs; g.y *= gs; g.z *= gs; g.w *= gs;
      adam_update(p.x, g.x, m.x, v.x, b1, b2, eps, decay, step_size, bc2_sqrt);
      adam_update(p.y, g.y, m.y, v.y, b1, b2, eps, decay, step_size, bc2_sqrt);
      adam_update(p.z, g.z, m.z, v.z, b1, b2, eps, decay, step_size, bc2_sqrt);
      adam_update(p.w, g.w, m.w, v.w, b1, b2, eps, decay, step_size, bc2_sqrt);
      p4[i] = p;
      m4[i] = m;
      v4[i] = v;
      if (copy) {
        __nv_bfloat162 lo = __floats2bfloat162_rn(p.x, p.y), hi = __floats2bfloat162_rn(p.z, p.w);
        const uint2 w = make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
        if (c4) c4[i] = w;
        // all-gather fused into the update: the new weights go straight to every rank's buffer
        if (c.peer_off >= 0)
          for (int j = 0; j < peers.n; ++j) reinterpret_cast<uint2*>(peers.base[j] + c.peer_off)[i] = w;
      }
    }
    return;
  }
  for (int i = threadIdx.x; i < c.n; i += NT) {
    const float g = ldv(c.g, i, c.g_bf16) * gs;
    float m = c.m[i], v = c.v[i];
    float pv = c.p_bf16 ? __bfloat162float(static_cast<__nv_bfloat16*>(c.p)[i]) : static_cast<float*>(c.p)[i];
    adam_update(pv, g, m, v, b1, b2, eps, decay, step_size, bc2_sqrt);
    c.m[i] = m;
    c.v[i] = v;
    if (c.p_bf16) static_cast<__nv_bfloat16*>(c.p)[i] = __float2bfloat16(pv);
    else static_cast<float*>(c.p)[i] = pv;
    if (c.p_copy) c.p_copy[i] = __float2bfloat16(pv);
    for (int j = 0; j < peers.n && c.peer_off >= 0; ++j) peers.base[j][c.peer_off + i] = __float2bfloat16(pv);
  }
}

// chunk table as a kernel argument (small updates)
__global__ void __launch_bounds__(NT) adamw_kernel(const __grid_constant__ Table t, float lr, float b1, float b2,
                                                   float eps, float wd, float bc1, float bc2_sqrt,
                                                   const float* __restrict__ clip_total, float clip_max,
                                                   const __grid_constant__ Peers peers) {
  adamw_chunk(t.c[blockIdx.x], lr, b1, b2, eps, wd, bc1, bc2_sqrt, clip_total, clip_max, peers);
}

// chunk table in device memory, one persistent grid striding over it (whole-model updates:
// one launch instead of one per 560 chunks, so no launch gaps or per-launch tails)
__global__ void __launch_bounds__(NT) adamw_table_kernel(const Chunk* __restrict__ tab, int n, float lr, float b1,
                                                         float b2, float eps, float wd, float bc1, float bc2_sqrt,
                                                         const float* __restrict__ clip_total, float clip_max,
                                                         const __grid_constant__ Peers peers) {
  for (int k = blockIdx.x; k < n; k += gridDim.x) {
    const Chunk c = tab[k];
    adamw_chunk(c, lr, b1, b2, eps, wd, bc1, bc2_sqrt, clip_total, clip_max, peers);
  }
}

// ---- gradient clipping: sum of squares over many tensors, then in-place scale
struct SqChunk {
  const void* x;
  int n;
  int8_t bf16;
  int8_t vec4;
};
struct SqTable {
  SqChunk c[MAX_CHUNKS];
  int base;  // index of this launch's first chunk in the partials array
};

__device__ __forceinline__ float sumsq_chunk(const SqChunk& c) {
  float acc = 0.f;
  if (c.vec4 && !c.bf16) {
    const float4* x4 = static_cast<const float4*>(c.x);
    for (int i = threadIdx.x; i < c.n / 4; i += NT) {
      const float4 v = x4[i];
      acc += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
  } else if (c.vec4) {  // bf16, four per 8-byte load
    const uint2* x4 = static_cast<const uint2*>(c.x);
    for (int i = threadIdx.x; i < c.n / 4; i += NT) {
      const uint2 r = x4[i];
      const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&r.x));
      const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&r.y));
      acc += a.x * a.x + a.y * a.y + b.x * b.x + b.y * b.y;
    }
  } else {
    for (int i = threadIdx.x; i < c.n; i += NT) {
      const float v = ldv(c.x, i, c.bf16);
      acc += v * v;
    }
  }
  return acc;
}

__device__ __forceinline__ void block_sum_store(float acc, float* out) {
#pragma unroll
  for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  __shared__ float sh[NT / 32];
  if (threadIdx.x % 32 == 0) sh[threadIdx.x / 32] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    acc = threadIdx.x < NT / 32 ? sh[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (threadIdx.x == 0) *out = acc;
  }
}

// device-table variant: each block sums its fixed set of chunks (k = blockIdx.x + j * gridDim.x),
// so the partials and their reduction order are the same run to run
__global__ void __launch_bounds__(NT) sumsq_table_kernel(const SqChunk* __restrict__ tab, int n,
                                                         float* __restrict__ partial) {
  float acc = 0.f;
  for (int k = blockIdx.x; k < n; k += gridDim.x) acc += sumsq_chunk(tab[k]);
  block_sum_store(acc, partial + blockIdx.x);
}

__global__ void __launch_bounds__(NT) sumsq_kernel(const __grid_constant__ SqTable t, float* __restrict__ partial) {
  const SqChunk c = t.c[blockIdx.x];
  float acc = sumsq_chunk(c);
#pragma unroll
  for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  __shared__ float sh[NT / 32];
  if (threadIdx.x % 32 == 0) sh[threadIdx.x / 32] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    acc = threadIdx.x < NT / 32 ? sh[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (threadIdx.x == 0) partial[t.base + blockIdx.x] = acc;
  }
}

__global__ void reduce_partials_kernel(const float* __restrict__ partial, int n, float* __restrict__ out) {
  __shared__ double sh[32];
  double acc = 0.0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) acc += partial[i];
#pragma unroll
  for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (threadIdx.x % 32 == 0) sh[threadIdx.x / 32] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    acc = threadIdx.x < blockDim.x / 32 ? sh[threadIdx.x] : 0.0;
#pragma unroll
    for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (threadIdx.x == 0) out[0] = static_cast<float>(acc);
  }
}

// x *= clamp(max_norm / (sqrt(total) + 1e-6), max=1); total read on the device
__global__ void __launch_bounds__(NT) clip_scale_kernel(const __grid_constant__ SqTable t, const float* __restrict__ total,
                                                        float max_norm) {
  const SqChunk c = t.c[blockIdx.x];
  const float coef = fminf(max_norm / (sqrtf(*total) + 1e-6f), 1.f);
  if (coef >= 1.f) return;
  if (c.vec4 && !c.bf16) {
    float4* x4 = static_cast<float4*>(const_cast<void*>(c.x));
    for (int i = threadIdx.x; i < c.n / 4; i += NT) {
      float4 v = x4[i];
      v.x *= coef; v.y *= coef; v.z *= coef; v.w *= coef;
      x4[i] = v;
    }
  } else if (c.bf16) {
    __nv_bfloat16* x = static_cast<__nv_bfloat16*>(const_cast<void*>(c.x));
    for (int i = threadIdx.x; i < c.n; i += NT) x[i] = __float2bfloat16(__bfloat162float(x[i]) * coef);
  } else {
    float* x = static_cast<float*>(const_cast<void*>(c.x));
    for (int i = threadIdx.x; i < c.n; i += NT) x[i] *= coef;
  }
}

}  // namespace

namespace {
// A chunk table kept in device memory per device, rebuilt and re-uploaded only when the tensor
// set changes (the parameters, optimizer state and gradient buffers normally keep their storage
// from step to step, so the upload happens once).
struct DevTable {
  uint64_t key = 0;
  void* dev = nullptr;
  size_t cap = 0;
  int n = 0;
};
constexpr int kMaxDev = 16;
DevTable g_adam_tab[kMaxDev], g_sq_tab[kMaxDev];

uint64_t fnv(uint64_t h, const void* p, size_t n) {
  const unsigned char* b = static_cast<const unsigned char*>(p);
  for (size_t i = 0; i < n; ++i) h = (h ^ b[i]) * 1099511628211ull;
  return h;
}

template <class T>
const T* device_table(DevTable* tabs, uint64_t key, int n, cudaStream_t s, const std::function<void(std::vector<T>&)>& build) {
  int dev = 0;
  check_cuda(cudaGetDevice(&dev), "adamw device");
  DevTable& t = tabs[dev % kMaxDev];
  if (t.key == key && t.n == n && t.dev != nullptr) return static_cast<const T*>(t.dev);
  std::vector<T> host;
  host.reserve(n);
  build(host);
  const size_t bytes = host.size() * sizeof(T);
  if (bytes > t.cap) {
    if (t.dev != nullptr) check_cuda(cudaFree(t.dev), "chunk table free");
    check_cuda(cudaMalloc(&t.dev, bytes), "chunk table alloc");
    t.cap = bytes;
  }
  // stream-ordered after every earlier kernel that read the old table; pageable source, so the
  // copy is staged before this call returns and the host vector may go away
  check_cuda(cudaMemcpyAsync(t.dev, host.data(), bytes, cudaMemcpyHostToDevice, s), "chunk table upload");
  t.key = key;
  t.n = n;
  return static_cast<const T*>(t.dev);
}

int persistent_blocks(const void* kernel) {
  int dev = 0, sms = 0, per_sm = 0;
  check_cuda(cudaGetDevice(&dev), "device");
  check_cuda(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "SM count");
  check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, NT, 0), "occupancy");
  return sms * (per_sm > 0 ? per_sm : 1);
}
}  // namespace

void adamw_multi(const AdamWTensor* list, int count, float lr, float beta1, float beta2, float eps, float wd, int step,
                 cudaStream_t s, const float* clip_total, float clip_max, void* const* peer_bases, int n_peers) {
  Peers peers;
  peers.n = n_peers;
  for (int j = 0; j < 8; ++j) peers.base[j] = j < n_peers ? static_cast<__nv_bfloat16*>(peer_bases[j]) : nullptr;
  const double bc1 = 1.0 - std::pow(static_cast<double>(beta1), step);
  const double bc2 = 1.0 - std::pow(static_cast<double>(beta2), step);
  auto make_chunk = [](const AdamWTensor& t, int64_t off) {
    Chunk c;
    const int esz_p = t.p_dtype ? 2 : 4, esz_g = t.g_dtype ? 2 : 4;
    c.p = static_cast<char*>(t.p) + off * esz_p;
    c.g = static_cast<const char*>(t.g) + off * esz_g;
    c.m = t.m + off;
    c.v = t.v + off;
    c.n = static_cast<int>(t.n - off < CHUNK ? t.n - off : CHUNK);
    c.p_bf16 = static_cast<int8_t>(t.p_dtype);
    c.g_bf16 = static_cast<int8_t>(t.g_dtype);
    c.p_copy = t.p_copy ? static_cast<__nv_bfloat16*>(t.p_copy) + off : nullptr;
    c.peer_off = t.peer_off >= 0 ? t.peer_off + off : -1;
    c.vec4 = static_cast<int8_t>(((reinterpret_cast<uintptr_t>(c.p) | reinterpret_cast<uintptr_t>(c.m) |
                                   reinterpret_cast<uintptr_t>(c.v)) & 15) == 0 &&
                                 (reinterpret_cast<uintptr_t>(c.g) & (t.g_dtype ? 7 : 15)) == 0 &&
                                 (reinterpret_cast<uintptr_t>(c.p_copy) & 7) == 0 && c.n % 4 == 0 &&
                                 (c.peer_off < 0 || c.peer_off % 4 == 0));
    return c;
  };
  int64_t total = 0;
  uint64_t key = 1469598103934665603ull;
  for (int i = 0; i < count; ++i) {
    total += (list[i].n + CHUNK - 1) / CHUNK;
    const AdamWTensor& t = list[i];  // field by field (no padding bytes in the key)
    key = fnv(key, &t.p, sizeof(t.p));
    key = fnv(key, &t.g, sizeof(t.g));
    key = fnv(key, &t.m, sizeof(t.m));
    key = fnv(key, &t.v, sizeof(t.v));
    key = fnv(key, &t.n, sizeof(t.n));
    key = fnv(key, &t.p_dtype, sizeof(t.p_dtype));
    key = fnv(key, &t.g_dtype, sizeof(t.g_dtype));
    key = fnv(key, &t.p_copy, sizeof(t.p_copy));
    key = fnv(key, &t.peer_off, sizeof(t.peer_off));
  }
  if (total > MAX_CHUNKS && total < (1 << 30)) {
    const Chunk* tab = device_table<Chunk>(g_adam_tab, key, static_cast<int>(total), s, [&](std::vector<Chunk>& v) {
      for (int i = 0; i < count; ++i)
        for (int64_t off = 0; off < list[i].n; off += CHUNK) v.push_back(make_chunk(list[i], off));
    });
    const int grid = static_cast<int>(std::min<int64_t>(total, persistent_blocks(reinterpret_cast<const void*>(
                                                                   adamw_table_kernel))));
    adamw_table_kernel<<<grid, NT, 0, s>>>(tab, static_cast<int>(total), lr, beta1, beta2, eps, wd,
                                            static_cast<float>(bc1), static_cast<float>(std::sqrt(bc2)), clip_total,
                                            clip_max, peers);
    check_cuda(cudaGetLastError(), "adamw (table)");
    return;
  }
  Table tab;
  int nc = 0;
  auto flush = [&]() {
    if (nc == 0) return;
    adamw_kernel<<<nc, NT, 0, s>>>(tab, lr, beta1, beta2, eps, wd, static_cast<float>(bc1),
                                   static_cast<float>(std::sqrt(bc2)), clip_total, clip_max, peers);
    check_cuda(cudaGetLastError(), "adamw");
    nc = 0;
  };
  for (int i = 0; i < count; ++i) {
    for (int64_t off = 0; off < list[i].n; off += CHUNK) {
      tab.c[nc] = make_chunk(list[i], off);
      if (++nc == MAX_CHUNKS) flush();
    }
  }
  flush();
}

namespace {
template <class F>
void for_each_sq_batch(const SumSqTensor* list, int count, F&& fn) {
  SqTable tab;
  tab.base = 0;
  int nc = 0, total = 0;
  for (int i = 0; i < count; ++i) {
    const int esz = list[i].bf16 ? 2 : 4;
    for (int64_t off = 0; off < list[i].n; off += CHUNK) {
      SqChunk& c = tab.c[nc];
      c.x = static_cast<const char*>(list[i].x) + off * esz;
      c.n = static_cast<int>(list[i].n - off < CHUNK ? list[i].n - off : CHUNK);
      c.bf16 = static_cast<int8_t>(list[i].bf16);
      c.vec4 = static_cast<int8_t>((reinterpret_cast<uintptr_t>(c.x) & 15) == 0 && c.n % 4 == 0);
      ++total;
      if (++nc == MAX_CHUNKS) {
        fn(tab, nc);
        tab.base += nc;
        nc = 0;
      }
    }
  }
  if (nc) fn(tab, nc);
}
}  // namespace

int64_t sumsq_num_chunks(const SumSqTensor* list, int count) {
  int64_t n = 0;
  for (int i = 0; i < count; ++i) n += (list[i].n + CHUNK - 1) / CHUNK;
  return n;
}

void multi_sumsq(const SumSqTensor* list, int count, float* partial, float* out, cudaStream_t s) {
  int64_t total = sumsq_num_chunks(list, count);
  if (total > MAX_CHUNKS && total < (1 << 30)) {
    uint64_t key = 1469598103934665603ull;
    for (int i = 0; i < count; ++i) {  // field by field: the struct has padding
      key = fnv(key, &list[i].x, sizeof(list[i].x));
      key = fnv(key, &list[i].n, sizeof(list[i].n));
      key = fnv(key, &list[i].bf16, sizeof(list[i].bf16));
    }
    const SqChunk* tab = device_table<SqChunk>(g_sq_tab, key, static_cast<int>(total), s, [&](std::vector<SqChunk>& v) {
      for (int i = 0; i < count; ++i) {
        const int esz = list[i].bf16 ? 2 : 4;
        for (int64_t off = 0; off < list[i].n; off += CHUNK) {
          SqChunk c;
          c.x = static_cast<const char*>(list[i].x) + off * esz;
          c.n = static_cast<int>(list[i].n - off < CHUNK ? list[i].n - off : CHUNK);
          c.bf16 = static_cast<int8_t>(list[i].bf16);
          c.vec4 = static_cast<int8_t>((reinterpret_cast<uintptr_t>(c.x) & 15) == 0 && c.n % 4 == 0);
          v.push_back(c);
        }
      }
    });
    const int grid = static_cast<int>(std::min<int64_t>(total, persistent_blocks(reinterpret_cast<const void*>(
                                                                   sumsq_table_kernel))));
    sumsq_table_kernel<<<grid, NT, 0, s>>>(tab, static_cast<int>(total), partial);
    reduce_partials_kernel<<<1, 1024, 0, s>>>(partial, grid, out);
    check_cuda(cudaGetLastError(), "multi_sumsq (table)");
    return;
  }
  int n = 0;
  for_each_sq_batch(list, count, [&](const SqTable& t, int nc) {
    sumsq_kernel<<<nc, NT, 0, s>>>(t, partial);
    n = t.base + nc;
  });
  reduce_partials_kernel<<<1, 1024, 0, s>>>(partial, n, out);
  check_cuda(cudaGetLastError(), "multi_sumsq");
}

void multi_clip_scale(const SumSqTensor* list, int count, const float* total, float max_norm, cudaStream_t s) {
  for_each_sq_batch(list, count, [&](const SqTable& t, int nc) {
    clip_scale_kernel<<<nc, NT, 0, s>>>(t, total, max_norm);
  });
  check_cuda(cudaGetLastError(), "multi_clip_scale");
}

}  // namespace ttb
