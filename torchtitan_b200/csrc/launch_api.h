// Plain C++ launch interface of the sm_100a kernels (no torch headers), so
// the .cu translation units compile quickly; tensor checks and allocation
// live in bindings.cpp.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <stdexcept>
#include <string>

namespace ttb {

inline void check_cuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

inline int num_sms(int dev) {
  static int cache[64] = {0};
  if (dev >= 0 && dev < 64 && cache[dev]) return cache[dev];
  int n = 0;
  check_cuda(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev), "sm count");
  if (dev >= 0 && dev < 64) cache[dev] = n;
  return n;
}

// gemm_tcgen05.cu
void gemm_bf16(const void* A, const void* B, void* D, int64_t M, int64_t N, int64_t K, bool a_mn, bool b_mn,
               cudaStream_t stream);
int gemm_error_code(bool reset);
// gemm_2sm.cu: same contract as gemm_bf16 on CTA pairs (256x256 tiles)
void gemm_bf16_2sm(const void* A, const void* B, void* D, int64_t M, int64_t N, int64_t K, bool a_mn, bool b_mn,
                   cudaStream_t stream);
int gemm2_error_code(bool reset);
// mode 1: per-M-tile group (tile_group[m_tile], -1 = skip) picks B rows [g*b_group_rows, ...);
// mode 2: group g reduces over K rows [kstart[g], kstart[g]+klen[g]) into D[g] (A, B M/N-major).
void gemm_bf16_grouped(const void* A, const void* B, void* D, int64_t M, int64_t N, int64_t K, bool a_mn,
                       bool b_mn, int mode, int num_groups, const int* tile_group, const int* kstart,
                       const int* klen, int64_t b_total_rows, int b_group_rows, cudaStream_t stream);

// elementwise.cu
void rmsnorm_fwd(const void* x, const void* w, void* y, float* rstd, int64_t rows, int64_t dim, float eps, int w_fp32,
                 cudaStream_t s);
void rmsnorm_bwd(const void* dy, const void* x, const void* w, const float* rstd, void* dx, float* dw_partial,
                 int64_t rows, int64_t dim, int w_fp32, int nparts, cudaStream_t s);
// out[p] = src[idx[p]] or a zero row where idx[p] < 0 (bf16, row length a multiple of 8)
void gather_rows_bf16(const void* src, int64_t n_src, const int64_t* idx, void* out, int64_t rows, int64_t d,
                      cudaStream_t s);
// moe_combine.cu: deterministic MoE combine (per-token gather-sum of the routed rows) and backward
void moe_combine_fwd(const void* base, const void* y, const int64_t* pos, const float* w, void* out, int64_t T,
                     int k, int64_t D, int64_t R, cudaStream_t s);
void moe_combine_bwd(const void* dout, const void* y, const int64_t* pos, const int64_t* token_of,
                     const float* scale, void* dy, float* dw, int64_t T, int k, int64_t D, int64_t R,
                     cudaStream_t s);
int rmsnorm_bwd_parts(int64_t rows, int64_t dim, int sms);
void reduce_rows_f32(const float* partial, float* out, int64_t nparts, int64_t dim, cudaStream_t s);
void rope_apply(const void* x, void* y, const float* cos, const float* sin, int64_t B, int64_t S, int64_t H,
                int64_t D, int64_t cs_batch_stride, bool inverse, cudaStream_t s);
void swiglu_fwd(const void* a, const void* b, void* y, int64_t n, cudaStream_t s);
void swiglu_bwd(const void* dy, const void* a, const void* b, void* da, void* db, int64_t n, cudaStream_t s);

// cross_entropy.cu
void ce_fwd(const void* logits, const int64_t* labels, float* loss_rows, float* lse, float* loss_sum, int64_t T,
            int64_t V, int64_t ignore_index, cudaStream_t s);
void ce_bwd(const void* logits, const int64_t* labels, const float* lse, const float* gscale, void* dlogits, int64_t T,
            int64_t V, int64_t ignore_index, cudaStream_t s);

// adamw.cu
struct AdamWTensor {
  void* p;
  const void* g;
  float* m;
  float* v;
  int64_t n;
  int p_dtype;  // 0 fp32, 1 bf16
  int g_dtype;
  void* p_copy = nullptr;  // optional bf16 copy of the updated fp32 param (compute weights)
  int64_t peer_off = -1;   // >= 0: write the bf16 copy at this offset of every peer weight buffer
};
void adamw_multi(const AdamWTensor* host_list, int count, float lr, float beta1, float beta2, float eps, float wd,
                 int step, cudaStream_t s, const float* clip_total = nullptr, float clip_max = 0.f,
                 void* const* peer_bases = nullptr, int n_peers = 0);

// dp_comm.cu: data-parallel collectives over NVLink peer memory
void dp_reduce_scatter_bucket(const void* const* peer_grads, uint32_t* const* peer_sigs, int world, int rank,
                              int64_t bucket_off, int64_t bucket_len, float* out_shard, float scale, int slot,
                              uint32_t epoch, int num_ctas, cudaStream_t s, double limit_s = 0.0);
void dp_barrier(uint32_t* const* peer_sigs, int world, int rank, int slot, uint32_t epoch, cudaStream_t s,
                double limit_s = 0.0);
int dp_error_code(bool reset);
void dp_set_error_sink(void* host_mapped_int8);  // pinned host int[8] written on the first wait failure
void dp_error_info(int* out4);

// gemm_mxfp8.cu / mx_quant.cu: MXFP8 block-scaled GEMM and its quantizer
// Optional epilogue scales of the block-scaled GEMM: D[m, n] *= sa[m] (or sa[0]) * sb[n] (or
// sb[0]); null pointers mean 1. Null scale records (sfa = sfb = nullptr) mean E8M0 2^0
// everywhere, which turns the kernel into a plain FP8 GEMM (Float8 tensorwise / rowwise).
struct MxEpilogue {
  const float* sa = nullptr;
  const float* sb = nullptr;
  int sa_rows = 0, sb_rows = 0;
  // grouped rows (routed experts): M-tile tm multiplies B rows [g*N, g*N + N) with
  // g = tile_group[tm]; g < 0 skips the tile (its output rows are left unwritten)
  const int* tile_group = nullptr;
  int num_groups = 1;
};
void gemm_mxfp8(const void* A, const void* B, const void* sfa, const void* sfb, void* D, int64_t M, int64_t N,
                int64_t K, cudaStream_t stream, int tile_n = 0, const MxEpilogue& ep = MxEpilogue());
// Float8 (E4M3) quantization along rows: scale = 448 / max(amax, 1e-12) per row (rowwise) or
// per tensor; writes codes [R, Cp] (columns zero padded to 128) and inv = 1 / scale ([R] or [1]).
void f8_quantize(const void* x, int64_t R, int64_t C, int64_t ldx, bool rowwise, void* codes, float* inv,
                 unsigned int* amax_word, cudaStream_t s);
int mxgemm_error_code(bool reset);
void mx_quantize(const void* x, int64_t R, int64_t C, int64_t ldx, void* codes, void* sf, cudaStream_t s);

// kda_gram.cu: decayed Gram matrices of chunked KDA (forward and backward)
void kda_gram_fwd(const float* a, const float* b, const float* G, float* out, int64_t N, int C, int K, bool strict,
                  cudaStream_t s);
void kda_gram_bwd(const float* dout, const float* a, const float* b, const float* G, float* da, float* db,
                  float* dG, int64_t N, int C, int K, bool strict, cudaStream_t s);

// kda_state.cu: the chunked-KDA state recurrence on tcgen05 (C = 64, K = V = 128, bf16 operands)
// kda_prep.cu: chunk preparation of the chunked KDA (layouts and formulas in the file)
void kda_prep_fwd(const float* q, const float* k, const float* g, int B, int T, int H, int K, int C, float* qc,
                  float* kc, float* G, float* kg, float* qg, float* kd, float* decay, cudaStream_t s);
void kda_prep_bwd(const float* q, const float* k, const float* G, int B, int T, int H, int K, int C,
                  const float* dqc, const float* dkc, const float* dG, const float* dkg, const float* dqg,
                  const float* dkd, const float* ddecay, float* dq, float* dk, float* dg, cudaStream_t s);
void kda_state_fwd(const void* w, const void* kd, const void* uT, const float* dec, const float* S0, void* states,
                   void* vnT, float* Sfin, int BH, int NT, cudaStream_t s);
void kda_state_bwd(const void* qg, const void* w, const void* kd, const void* dO, const void* Aqk, const float* dec,
                   const float* dSfin, void* dstates, float* duT, float* dS0, int BH, int NT, cudaStream_t s);
int kda_state_error_code(bool reset);

// kda_scan.cu: inter-chunk state recurrence of chunked KDA (forward and backward)
void kda_scan_fwd(const float* u, const float* w, const float* qg, const float* Aqk, const float* kdec,
                  const float* dec, float* o, float* states, float* final_S, int64_t BH, int NT, int C, int K, int V,
                  int VS, cudaStream_t s);
void kda_scan_bwd(const float* dO, const float* u, const float* w, const float* qg, const float* Aqk,
                  const float* kdec, const float* dec, const float* states, float* du, float* p_dqg, float* p_dw,
                  float* p_dkdec, float* p_dA, float* p_dd, int64_t BH, int NT, int C, int K, int V, int VS,
                  cudaStream_t s);

// attn_res.cu: block attention-residual mixing (forward and backward), blocks read in place
void attn_res_fwd(const void* const* blocks, int nb, const float* u, void* out, int64_t T, int D, float eps,
                  cudaStream_t s);
void attn_res_bwd(const void* const* blocks, void* const* dblocks, int nb, const float* u, const void* dout, float* du,
                  int64_t T, int D, float eps, cudaStream_t s);

// kda_eltwise.cu: KDA short causal conv + SiLU and gated RMSNorm (forward and backward)
void kda_short_conv_fwd(const void* x, const float* w, void* y, int64_t B, int64_t T, int C, int W, cudaStream_t s);
void kda_short_conv_bwd(const void* x, const float* w, const void* dy, void* dx, float* dw, int64_t B, int64_t T,
                        int C, int W, cudaStream_t s);
void kda_gated_norm_fwd(const void* x, const void* z, const float* g, void* y, int64_t R, int D, float eps,
                        cudaStream_t s);
void kda_gated_norm_bwd(const void* x, const void* z, const float* g, const void* dy, void* dx, void* dz, float* dg,
                        int64_t R, int D, float eps, cudaStream_t s);
void kda_gate_fwd(const void* x, const float* A, const float* b, float* g, int64_t n, int H, int K, cudaStream_t s);
void kda_gate_bwd(const void* x, const float* A, const float* b, const float* dg, void* dx, float* dA, float* db,
                  int64_t n, int H, int K, cudaStream_t s);

// router_topk.cu: MoE routing selection (scores, bias, group limit, top-k, counts)
void router_topk(const float* logits, const float* bias, int64_t T, int E, int top_k, bool sigmoid, int n_groups,
                 int n_limited, int64_t* idx, int32_t* counts, cudaStream_t s);

// ep_comm.cu: expert-parallel row movement over NVLink peer memory
void ep_scatter_rows(const void* src, int64_t n, int d, const int32_t* dest_rank, const int64_t* dest_row,
                     void* const* peer_bases, int world, int64_t cap_rows, cudaStream_t s);
void ep_gather_rows(void* dst, int64_t n, int d, const int32_t* src_rank, const int64_t* src_row,
                    void* const* peer_bases, int world, int64_t cap_rows, cudaStream_t s);
int ep_error_code(bool reset);

// tp_gemm.cu: tensor-parallel GEMMs fused with their all-gather / reduce-scatter over peer memory
void tp_gemm(int mode, const void* const* shards, void* land, unsigned* chunk_ready, void* D, const void* B, bool b_mn,
             void* const* recv, unsigned* const* done, void* out, int parity, unsigned* const* sig, int tp, int rank,
             uint32_t epoch, int64_t Ms, int64_t N, int64_t K, cudaStream_t s);
int tp_gemm_error_code(bool reset);  // slot, epoch, source rank, flag value of the first failed wait

struct SumSqTensor {
  const void* x;
  int64_t n;
  int bf16;
};
int64_t sumsq_num_chunks(const SumSqTensor* list, int count);
// partial: >= sumsq_num_chunks floats of scratch; out: 1 float (sum of squares)
void multi_sumsq(const SumSqTensor* list, int count, float* partial, float* out, cudaStream_t s);
// scale every tensor by min(1, max_norm / (sqrt(*total) + 1e-6)) with *total read on the device
void multi_clip_scale(const SumSqTensor* list, int count, const float* total, float max_norm, cudaStream_t s);

// flash_attn.cu
void attn_fwd(const void* q, const void* k, const void* v, void* o, float* lse, int B, int Sq, int Sk, int H, int Hk,
              int Dqk, int Dv, bool causal, float scale, cudaStream_t s, const int* doc_start = nullptr,
              const int* doc_end = nullptr);
void attn_bwd(const void* dout, const void* q, const void* k, const void* v, const void* o, const float* lse,
              void* dq, void* dk, void* dv, float* dq_acc, float* delta, int B, int Sq, int Sk, int H, int Hk,
              int Dqk, int Dv, bool causal, float scale, cudaStream_t s, const float* dlse = nullptr,
              const int* doc_start = nullptr, const int* doc_end = nullptr);
int attn_error_code(bool reset);

}  // namespace ttb
