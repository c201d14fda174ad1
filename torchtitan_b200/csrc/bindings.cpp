// Python bindings of the sm_100a kernels: argument checks, output allocation
// through the caching allocator, current-stream launch.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <vector>

#include "launch_api.h"

namespace {

using torch::Tensor;

cudaStream_t stream() { return at::cuda::getCurrentCUDAStream(); }

void check_cuda_bf16(const Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.scalar_type() == at::kBFloat16, name, " must be bfloat16");
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}

Tensor gemm(Tensor A, Tensor B, bool a_mn, bool b_mn) {
  check_cuda_bf16(A, "A");
  check_cuda_bf16(B, "B");
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2, "gemm: 2-D operands required");
  c10::cuda::CUDAGuard g(A.device());
  const int64_t M = a_mn ? A.size(1) : A.size(0), K = a_mn ? A.size(0) : A.size(1);
  const int64_t N = b_mn ? B.size(1) : B.size(0), Kb = b_mn ? B.size(0) : B.size(1);
  TORCH_CHECK(K == Kb, "gemm: reduction dims differ (", K, " vs ", Kb, ")");
  Tensor D = torch::empty({M, N}, A.options());
  ttb::gemm_bf16(A.data_ptr(), B.data_ptr(), D.data_ptr(), M, N, K, a_mn, b_mn, stream());
  return D;
}

Tensor gemm_2sm(Tensor A, Tensor B, bool a_mn, bool b_mn) {
  check_cuda_bf16(A, "A");
  check_cuda_bf16(B, "B");
  c10::cuda::CUDAGuard g(A.device());
  const int64_t M = a_mn ? A.size(1) : A.size(0), K = a_mn ? A.size(0) : A.size(1);
  const int64_t N = b_mn ? B.size(1) : B.size(0), Kb = b_mn ? B.size(0) : B.size(1);
  TORCH_CHECK(K == Kb, "gemm_2sm: reduction dims differ");
  TORCH_CHECK((a_mn ? M : K) % 8 == 0 && (b_mn ? N : K) % 8 == 0, "gemm_2sm: contiguous dims must be multiples of 8");
  Tensor D = torch::empty({M, N}, A.options());
  if (M > 0 && N > 0 && K > 0) ttb::gemm_bf16_2sm(A.data_ptr(), B.data_ptr(), D.data_ptr(), M, N, K, a_mn, b_mn, stream());
  return D;
}

// mode 1 (grouped rows): A [Mp, K] padded rows, B [G*N, K] (or [G*K, N] if b_mn), tile_group [Mp/128] int32
Tensor gemm_grouped_rows(Tensor A, Tensor B, Tensor tile_group, int64_t n_out, int64_t b_group_rows, bool b_mn) {
  check_cuda_bf16(A, "A");
  check_cuda_bf16(B, "B");
  TORCH_CHECK(tile_group.scalar_type() == at::kInt && tile_group.is_contiguous(), "tile_group int32");
  c10::cuda::CUDAGuard g(A.device());
  const int64_t M = A.size(0), K = A.size(1);
  TORCH_CHECK(M % 128 == 0 && tile_group.numel() == M / 128, "padded rows must be a multiple of 128");
  Tensor D = torch::empty({M, n_out}, A.options());
  ttb::gemm_bf16_grouped(A.data_ptr(), B.data_ptr(), D.data_ptr(), M, n_out, K, false, b_mn, 1, 1,
                         tile_group.data_ptr<int>(), nullptr, nullptr, B.size(0), (int)b_group_rows, stream());
  return D;
}

// mode 2 (grouped reduction): A [Ktot, M], B [Ktot, N]; D [G, M, N]; kstart/klen int32 [G]
Tensor gemm_grouped_k(Tensor A, Tensor B, Tensor kstart, Tensor klen) {
  check_cuda_bf16(A, "A");
  check_cuda_bf16(B, "B");
  c10::cuda::CUDAGuard g(A.device());
  const int64_t G = kstart.numel(), M = A.size(1), N = B.size(1), Ktot = A.size(0);
  TORCH_CHECK(B.size(0) == Ktot, "grouped K: row counts differ");
  Tensor D = torch::empty({G, M, N}, A.options());
  ttb::gemm_bf16_grouped(A.data_ptr(), B.data_ptr(), D.data_ptr(), M, N, Ktot, true, true, 2, (int)G, nullptr,
                         kstart.data_ptr<int>(), klen.data_ptr<int>(), Ktot, 0, stream());
  return D;
}

std::vector<Tensor> rmsnorm_fwd(Tensor x, Tensor w, double eps) {
  check_cuda_bf16(x, "x");
  TORCH_CHECK(x.dim() == 2 && w.dim() == 1 && w.size(0) == x.size(1), "rmsnorm: shape mismatch");
  TORCH_CHECK(w.is_contiguous() && (w.scalar_type() == at::kBFloat16 || w.scalar_type() == at::kFloat),
              "rmsnorm: weight must be contiguous bf16/fp32");
  c10::cuda::CUDAGuard g(x.device());
  Tensor y = torch::empty_like(x);
  Tensor rstd = torch::empty({x.size(0)}, x.options().dtype(at::kFloat));
  ttb::rmsnorm_fwd(x.data_ptr(), w.data_ptr(), y.data_ptr(), rstd.data_ptr<float>(), x.size(0), x.size(1),
                   static_cast<float>(eps), w.scalar_type() == at::kFloat, stream());
  return {y, rstd};
}

std::vector<Tensor> rmsnorm_bwd(Tensor dy, Tensor x, Tensor w, Tensor rstd) {
  check_cuda_bf16(dy, "dy");
  check_cuda_bf16(x, "x");
  c10::cuda::CUDAGuard g(x.device());
  Tensor dx = torch::empty_like(x);
  const int64_t rows = x.size(0), dim = x.size(1);
  int dev = x.get_device();
  const int nparts = ttb::rmsnorm_bwd_parts(rows, dim, ttb::num_sms(dev));
  Tensor part = torch::empty({nparts, dim}, x.options().dtype(at::kFloat));
  Tensor dw = torch::empty({dim}, x.options().dtype(at::kFloat));
  if (rows > 0) {
    ttb::rmsnorm_bwd(dy.data_ptr(), x.data_ptr(), w.data_ptr(), rstd.data_ptr<float>(), dx.data_ptr(),
                     part.data_ptr<float>(), rows, dim, w.scalar_type() == at::kFloat, nparts, stream());
    ttb::reduce_rows_f32(part.data_ptr<float>(), dw.data_ptr<float>(), nparts, dim, stream());
  } else {
    dw.zero_();
  }
  return {dx, dw};
}

Tensor rope(Tensor x, Tensor cos, Tensor sin, bool inverse) {
  check_cuda_bf16(x, "x");
  TORCH_CHECK(x.dim() == 4, "rope: x must be [B,S,H,D]");
  TORCH_CHECK(cos.scalar_type() == at::kFloat && sin.scalar_type() == at::kFloat, "rope: fp32 tables");
  cos = cos.contiguous();
  sin = sin.contiguous();
  const int64_t B = x.size(0), S = x.size(1), H = x.size(2), D = x.size(3);
  int64_t bstride = 0;
  if (cos.dim() == 3) {
    TORCH_CHECK(cos.size(0) == B && cos.size(1) == S && cos.size(2) == D / 2, "rope: table shape");
    bstride = S * (D / 2);
  } else {
    TORCH_CHECK(cos.dim() == 2 && cos.size(0) >= S && cos.size(1) == D / 2, "rope: table shape");
  }
  c10::cuda::CUDAGuard g(x.device());
  Tensor y = torch::empty_like(x);
  ttb::rope_apply(x.data_ptr(), y.data_ptr(), cos.data_ptr<float>(), sin.data_ptr<float>(), B, S, H, D, bstride,
                  inverse, stream());
  return y;
}

Tensor swiglu_fwd(Tensor a, Tensor b) {
  check_cuda_bf16(a, "a");
  check_cuda_bf16(b, "b");
  TORCH_CHECK(a.sizes() == b.sizes(), "swiglu: shape mismatch");
  c10::cuda::CUDAGuard g(a.device());
  Tensor y = torch::empty_like(a);
  ttb::swiglu_fwd(a.data_ptr(), b.data_ptr(), y.data_ptr(), a.numel(), stream());
  return y;
}

std::vector<Tensor> swiglu_bwd(Tensor dy, Tensor a, Tensor b) {
  check_cuda_bf16(dy, "dy");
  c10::cuda::CUDAGuard g(a.device());
  Tensor da = torch::empty_like(a), db = torch::empty_like(b);
  ttb::swiglu_bwd(dy.data_ptr(), a.data_ptr(), b.data_ptr(), da.data_ptr(), db.data_ptr(), a.numel(), stream());
  return {da, db};
}

std::vector<Tensor> ce_fwd(Tensor logits, Tensor labels, int64_t ignore_index) {
  check_cuda_bf16(logits, "logits");
  TORCH_CHECK(labels.scalar_type() == at::kLong && labels.is_contiguous(), "labels must be contiguous int64");
  TORCH_CHECK(logits.dim() == 2 && labels.numel() == logits.size(0), "ce: shape mismatch");
  c10::cuda::CUDAGuard g(logits.device());
  const int64_t T = logits.size(0), V = logits.size(1);
  auto f32 = logits.options().dtype(at::kFloat);
  Tensor rows = torch::empty({T}, f32), lse = torch::empty({T}, f32), loss = torch::empty({}, f32);
  ttb::ce_fwd(logits.data_ptr(), labels.data_ptr<int64_t>(), rows.data_ptr<float>(), lse.data_ptr<float>(),
              loss.data_ptr<float>(), T, V, ignore_index, stream());
  return {loss, lse};
}

Tensor ce_bwd(Tensor logits, Tensor labels, Tensor lse, Tensor gscale, int64_t ignore_index) {
  c10::cuda::CUDAGuard g(logits.device());
  Tensor d = torch::empty_like(logits);
  ttb::ce_bwd(logits.data_ptr(), labels.data_ptr<int64_t>(), lse.data_ptr<float>(), gscale.data_ptr<float>(),
              d.data_ptr(), logits.size(0), logits.size(1), ignore_index, stream());
  return d;
}

void adamw(std::vector<Tensor> params, std::vector<Tensor> grads, std::vector<Tensor> ms, std::vector<Tensor> vs,
           double lr, double b1, double b2, double eps, double wd, int64_t step, std::vector<Tensor> copies,
           c10::optional<Tensor> clip_total, double clip_max, std::vector<int64_t> peer_offsets,
           std::vector<int64_t> peer_bases) {
  TORCH_CHECK(peer_offsets.empty() || peer_offsets.size() == params.size(), "adamw: peer_offsets size");
  TORCH_CHECK(peer_bases.size() <= 8, "adamw: at most 8 peers");
  TORCH_CHECK(copies.empty() || copies.size() == params.size(), "adamw: copies must be empty or match params");
  TORCH_CHECK(params.size() == grads.size() && params.size() == ms.size() && params.size() == vs.size(),
              "adamw: list lengths differ");
  if (params.empty()) return;
  c10::cuda::CUDAGuard g(params[0].device());
  std::vector<ttb::AdamWTensor> list;
  list.reserve(params.size());
  for (size_t i = 0; i < params.size(); ++i) {
    auto &p = params[i], &gr = grads[i], &m = ms[i], &v = vs[i];
    TORCH_CHECK(p.is_cuda() && p.is_contiguous() && gr.is_contiguous() && m.is_contiguous() && v.is_contiguous(),
                "adamw: tensors must be contiguous CUDA tensors");
    TORCH_CHECK(m.scalar_type() == at::kFloat && v.scalar_type() == at::kFloat, "adamw: fp32 moments required");
    TORCH_CHECK(p.numel() == gr.numel() && p.numel() == m.numel() && p.numel() == v.numel(), "adamw: numel mismatch");
    TORCH_CHECK(p.scalar_type() == at::kFloat || p.scalar_type() == at::kBFloat16, "adamw: param fp32/bf16");
    TORCH_CHECK(gr.scalar_type() == at::kFloat || gr.scalar_type() == at::kBFloat16, "adamw: grad fp32/bf16");
    void* cp = nullptr;
    if (!copies.empty() && copies[i].defined() && copies[i].numel() > 0) {
      TORCH_CHECK(copies[i].scalar_type() == at::kBFloat16 && copies[i].is_contiguous() &&
                      copies[i].numel() == p.numel() && p.scalar_type() == at::kFloat,
                  "adamw: a copy must be a contiguous bf16 tensor of an fp32 param");
      cp = copies[i].data_ptr();
    }
    list.push_back({p.data_ptr(), gr.data_ptr(), m.data_ptr<float>(), v.data_ptr<float>(), p.numel(),
                    p.scalar_type() == at::kBFloat16 ? 1 : 0, gr.scalar_type() == at::kBFloat16 ? 1 : 0, cp,
                    peer_offsets.empty() ? -1 : peer_offsets[i]});
  }
  ttb::adamw_multi(list.data(), static_cast<int>(list.size()), static_cast<float>(lr), static_cast<float>(b1),
                   static_cast<float>(b2), static_cast<float>(eps), static_cast<float>(wd), static_cast<int>(step),
                   stream(), clip_total.has_value() ? clip_total->data_ptr<float>() : nullptr,
                   static_cast<float>(clip_max), reinterpret_cast<void* const*>(peer_bases.data()),
                   static_cast<int>(peer_bases.size()));
}

std::vector<ttb::SumSqTensor> sq_list(const std::vector<Tensor>& xs) {
  std::vector<ttb::SumSqTensor> l;
  l.reserve(xs.size());
  for (auto& x : xs) {
    TORCH_CHECK(x.is_cuda() && x.is_contiguous(), "grad norm: contiguous CUDA tensors required");
    TORCH_CHECK(x.scalar_type() == at::kFloat || x.scalar_type() == at::kBFloat16, "grad norm: fp32/bf16 only");
    l.push_back({x.data_ptr(), x.numel(), x.scalar_type() == at::kBFloat16 ? 1 : 0});
  }
  return l;
}

// sum of squares of all tensors (fp32 scalar tensor on the device)
Tensor multi_sumsq(std::vector<Tensor> xs) {
  TORCH_CHECK(!xs.empty(), "multi_sumsq: empty list");
  c10::cuda::CUDAGuard g(xs[0].device());
  auto l = sq_list(xs);
  const int64_t nchunks = std::max<int64_t>(1, ttb::sumsq_num_chunks(l.data(), (int)l.size()));
  auto opts = xs[0].options().dtype(at::kFloat);
  Tensor partial = torch::empty({nchunks}, opts);
  Tensor out = torch::empty({}, opts);
  ttb::multi_sumsq(l.data(), (int)l.size(), partial.data_ptr<float>(), out.data_ptr<float>(), stream());
  return out;
}

void multi_clip_scale(std::vector<Tensor> xs, Tensor total, double max_norm) {
  if (xs.empty()) return;
  c10::cuda::CUDAGuard g(xs[0].device());
  auto l = sq_list(xs);
  ttb::multi_clip_scale(l.data(), (int)l.size(), total.data_ptr<float>(), static_cast<float>(max_norm), stream());
}

// packed-document tables: int32 [B, S] on the device, contiguous
static const int* doc_table(const c10::optional<Tensor>& t, int64_t B, int64_t S) {
  if (!t.has_value()) return nullptr;
  TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kInt && t->is_contiguous() && t->numel() == B * S,
              "document table: contiguous int32 [B, S] on the device");
  return t->data_ptr<int>();
}

std::vector<Tensor> attn_fwd(Tensor q, Tensor k, Tensor v, bool causal, double scale,
                             c10::optional<Tensor> doc_start, c10::optional<Tensor> doc_end) {
  check_cuda_bf16(q, "q");
  check_cuda_bf16(k, "k");
  check_cuda_bf16(v, "v");
  TORCH_CHECK(q.dim() == 4 && k.dim() == 4 && v.dim() == 4, "attention: [B,S,H,D] tensors");
  const int B = q.size(0), Sq = q.size(1), H = q.size(2), Dqk = q.size(3);
  const int Sk = k.size(1), Hk = k.size(2), Dv = v.size(3);
  TORCH_CHECK(k.size(0) == B && v.size(0) == B && v.size(1) == Sk && v.size(2) == Hk && k.size(3) == Dqk,
              "attention: shape mismatch");
  TORCH_CHECK(H % Hk == 0, "attention: n_heads must be a multiple of n_kv_heads");
  c10::cuda::CUDAGuard g(q.device());
  Tensor o = torch::empty({B, Sq, H, Dv}, q.options());
  // rows padded to a multiple of 64 and zero-filled (the backward bulk-copies 64-query slices)
  Tensor lse = torch::zeros({B, H, (Sq + 63) / 64 * 64}, q.options().dtype(at::kFloat));
  ttb::attn_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr<float>(), B, Sq, Sk, H, Hk, Dqk,
                Dv, causal, static_cast<float>(scale), stream(), doc_table(doc_start, B, Sq),
                doc_table(doc_end, B, Sq));
  return {o, lse};
}

std::vector<Tensor> attn_bwd(Tensor dout, Tensor q, Tensor k, Tensor v, Tensor o, Tensor lse, bool causal,
                             double scale, c10::optional<Tensor> dlse, c10::optional<Tensor> doc_start,
                             c10::optional<Tensor> doc_end) {
  check_cuda_bf16(dout, "dout");
  const int B = q.size(0), Sq = q.size(1), H = q.size(2), Dqk = q.size(3);
  const int Sk = k.size(1), Hk = k.size(2), Dv = v.size(3);
  c10::cuda::CUDAGuard g(q.device());
  Tensor dq = torch::empty_like(q), dk = torch::empty_like(k), dv = torch::empty_like(v);
  Tensor delta = torch::zeros({B, H, (Sq + 63) / 64 * 64}, q.options().dtype(at::kFloat));
  if (dlse.has_value())
    TORCH_CHECK(dlse->is_cuda() && dlse->scalar_type() == at::kFloat && dlse->is_contiguous() &&
                    dlse->sizes() == delta.sizes(), "attn_bwd: dlse must be fp32 [B, H, padded Sq] like lse");
  ttb::attn_bwd(dout.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr<float>(),
                dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), nullptr, delta.data_ptr<float>(), B, Sq, Sk, H, Hk, Dqk,
                Dv, causal, static_cast<float>(scale), stream(),
                dlse.has_value() ? dlse->data_ptr<float>() : nullptr, doc_table(doc_start, B, Sq),
                doc_table(doc_end, B, Sq));
  return {dq, dk, dv};
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "torchtitan_b200 sm_100a kernels";
  m.def("gemm", &gemm, "bf16 GEMM on tcgen05: D = A(m,k) * B(n,k)");
  m.def("gemm_2sm", &gemm_2sm, "bf16 GEMM on tcgen05 CTA pairs (cta_group::2)");
  m.def("gemm2_error_code", &ttb::gemm2_error_code, py::arg("reset") = true);
  m.def("gemm_grouped_rows", &gemm_grouped_rows, "grouped GEMM over 128-row padded expert segments");
  m.def("gemm_grouped_k", &gemm_grouped_k, "grouped GEMM reducing over per-group row ranges (expert wgrad)");
  m.def("gemm_error_code", &ttb::gemm_error_code, "read (and optionally clear) the GEMM timeout word",
        py::arg("reset") = true);
  m.def("attn_error_code", &ttb::attn_error_code, "read (and optionally clear) the attention timeout word",
        py::arg("reset") = true);
  m.def("rmsnorm_fwd", &rmsnorm_fwd);
  m.def("rmsnorm_bwd", &rmsnorm_bwd);
  m.def("gather_rows", [](Tensor src, Tensor idx) {
    check_cuda_bf16(src, "src");
    TORCH_CHECK(src.dim() == 2 && src.is_contiguous() && idx.scalar_type() == at::kLong && idx.is_cuda() &&
                    idx.dim() == 1 && idx.is_contiguous(),
                "gather_rows: src [n, d] contiguous bf16, idx [rows] int64 (negative = zero row)");
    c10::cuda::CUDAGuard g(src.device());
    auto out = torch::empty({idx.size(0), src.size(1)}, src.options());
    ttb::gather_rows_bf16(src.data_ptr(), src.size(0), idx.data_ptr<int64_t>(), out.data_ptr(), idx.size(0), src.size(1),
                          stream());
    return out;
  });
  m.def("rope", &rope);
  m.def("swiglu_fwd", &swiglu_fwd);
  m.def("swiglu_bwd", &swiglu_bwd);
  m.def("ce_fwd", &ce_fwd);
  m.def("ce_bwd", &ce_bwd);
  m.def("adamw", &adamw, py::arg("params"), py::arg("grads"), py::arg("exp_avgs"), py::arg("exp_avg_sqs"),
        py::arg("lr"), py::arg("beta1"), py::arg("beta2"), py::arg("eps"), py::arg("weight_decay"), py::arg("step"),
        py::arg("copies") = std::vector<Tensor>(), py::arg("clip_total") = py::none(), py::arg("clip_max") = 0.0,
        py::arg("peer_offsets") = std::vector<int64_t>(), py::arg("peer_bases") = std::vector<int64_t>());
  m.def("dp_reduce_scatter_bucket", [](std::vector<int64_t> grads, std::vector<int64_t> sigs, int rank,
                                       int64_t off, int64_t len, Tensor out, double scale, int slot, int64_t epoch,
                                       int ctas, double limit_s) {
    TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kFloat && out.is_contiguous(), "out: fp32 CUDA");
    TORCH_CHECK((int64_t)grads.size() == (int64_t)sigs.size(), "grads / signal pads differ");
    c10::cuda::CUDAGuard g(out.device());
    ttb::dp_reduce_scatter_bucket(reinterpret_cast<const void* const*>(grads.data()),
                                  reinterpret_cast<uint32_t* const*>(sigs.data()), (int)grads.size(), rank, off, len,
                                  out.data_ptr<float>(), (float)scale, slot, (uint32_t)epoch, ctas, stream(),
                                  limit_s);
  });
  m.def(
      "dp_barrier",
      [](std::vector<int64_t> sigs, int rank, int slot, int64_t epoch, double limit_s) {
        ttb::dp_barrier(reinterpret_cast<uint32_t* const*>(sigs.data()), (int)sigs.size(), rank, slot,
                        (uint32_t)epoch, stream(), limit_s);
      },
      py::arg("sigs"), py::arg("rank"), py::arg("slot"), py::arg("epoch"), py::arg("limit_s") = 0.0);
  m.def("dp_error_code", &ttb::dp_error_code, py::arg("reset") = true);
  m.def("dp_set_error_sink", [](Tensor sink) {
    TORCH_CHECK(!sink.is_cuda() && sink.is_pinned() && sink.scalar_type() == at::kInt && sink.numel() >= 8,
                "sink: pinned host int32 tensor of >= 8 elements");
    ttb::dp_set_error_sink(sink.data_ptr());
  });
  m.def("ep_scatter_rows", [](Tensor src, Tensor dest_rank, Tensor dest_row, std::vector<int64_t> bases,
                              int64_t cap_rows) {
    check_cuda_bf16(src, "src");
    TORCH_CHECK(src.dim() == 2 && src.is_contiguous(), "src: contiguous [n, D]");
    TORCH_CHECK(dest_rank.scalar_type() == at::kInt && dest_row.scalar_type() == at::kLong, "index dtypes");
    TORCH_CHECK(dest_rank.numel() == src.size(0) && dest_row.numel() == src.size(0), "index lengths");
    c10::cuda::CUDAGuard g(src.device());
    ttb::ep_scatter_rows(src.data_ptr(), src.size(0), (int)src.size(1), dest_rank.data_ptr<int32_t>(),
                         dest_row.data_ptr<int64_t>(), reinterpret_cast<void* const*>(bases.data()),
                         (int)bases.size(), cap_rows, stream());
  });
  m.def("ep_gather_rows", [](Tensor dst, Tensor src_rank, Tensor src_row, std::vector<int64_t> bases,
                             int64_t cap_rows) {
    check_cuda_bf16(dst, "dst");
    TORCH_CHECK(dst.dim() == 2 && dst.is_contiguous(), "dst: contiguous [n, D]");
    TORCH_CHECK(src_rank.scalar_type() == at::kInt && src_row.scalar_type() == at::kLong, "index dtypes");
    TORCH_CHECK(src_rank.numel() == dst.size(0) && src_row.numel() == dst.size(0), "index lengths");
    c10::cuda::CUDAGuard g(dst.device());
    ttb::ep_gather_rows(dst.data_ptr(), dst.size(0), (int)dst.size(1), src_rank.data_ptr<int32_t>(),
                        src_row.data_ptr<int64_t>(), reinterpret_cast<void* const*>(bases.data()),
                        (int)bases.size(), cap_rows, stream());
  });
  // fused tensor-parallel GEMM (mode 0: all-gather -> GEMM, 1: GEMM -> reduce-scatter); pointers
  // of symmetric buffers as integers (every rank's mapping)
  m.def("tp_gemm", [](int64_t mode, std::vector<int64_t> shards, c10::optional<Tensor> land,
                      c10::optional<Tensor> ready, c10::optional<Tensor> D, Tensor B, bool b_mn,
                      std::vector<int64_t> recv, std::vector<int64_t> done, c10::optional<Tensor> out,
                      int64_t parity, std::vector<int64_t> sig, int64_t tp, int64_t rank, int64_t epoch, int64_t Ms,
                      int64_t N, int64_t K) {
    check_cuda_bf16(B, "B");
    TORCH_CHECK(B.is_contiguous(), "tp_gemm: B contiguous");
    TORCH_CHECK((int64_t)sig.size() == tp && (int64_t)shards.size() == tp, "tp_gemm: one pointer per rank");
    if (mode == 0) {
      TORCH_CHECK(land.has_value() && ready.has_value() && D.has_value(), "tp_gemm: ag buffers");
    } else {
      TORCH_CHECK(out.has_value() && (int64_t)recv.size() == tp && (int64_t)done.size() == tp, "tp_gemm: rs buffers");
    }
    c10::cuda::CUDAGuard g(B.device());
    auto vp = [](const std::vector<int64_t>& v) {
      std::vector<void*> r(v.size());
      for (size_t i = 0; i < v.size(); ++i) r[i] = reinterpret_cast<void*>(v[i]);
      return r;
    };
    auto sh = vp(shards), rc = vp(recv), dn = vp(done), sg = vp(sig);
    ttb::tp_gemm((int)mode, sh.data(), land.has_value() ? land->data_ptr() : nullptr,
                 ready.has_value() ? reinterpret_cast<unsigned*>(ready->data_ptr<int>()) : nullptr,
                 D.has_value() ? D->data_ptr() : nullptr, B.data_ptr(), b_mn, rc.data(),
                 reinterpret_cast<unsigned* const*>(dn.data()), out.has_value() ? out->data_ptr() : nullptr,
                 (int)parity, reinterpret_cast<unsigned* const*>(sg.data()), (int)tp, (int)rank,
                 static_cast<uint32_t>(epoch), Ms, N, K, stream());
  });
  m.def("tp_gemm_error_code", &ttb::tp_gemm_error_code, py::arg("reset") = true);
  m.def("ep_error_code", &ttb::ep_error_code, "read (and optionally clear) the EP out-of-capacity row flag",
        py::arg("reset") = true);
  m.def("mx_quantize", [](Tensor x) {
    check_cuda_bf16(x, "x");
    TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1, "mx_quantize: [R, C] with contiguous rows");
    const int64_t R = x.size(0), C = x.size(1);
    const int64_t Cp = (C + 127) / 128 * 128, Rp = (R + 127) / 128 * 128;
    c10::cuda::CUDAGuard g(x.device());
    auto codes = torch::empty({R, Cp}, x.options().dtype(at::kByte));
    auto sf = torch::empty({Rp * Cp / 32}, x.options().dtype(at::kByte));
    ttb::mx_quantize(x.data_ptr(), R, C, x.stride(0), codes.data_ptr(), sf.data_ptr(), stream());
    return std::vector<Tensor>{codes, sf};
  });
  m.def("gemm_mxfp8", [](Tensor a, Tensor sfa, Tensor b, Tensor sfb, int64_t tile_n) {
    TORCH_CHECK(a.is_cuda() && b.is_cuda() && a.scalar_type() == at::kByte && b.scalar_type() == at::kByte,
                "gemm_mxfp8: uint8 FP8 codes on CUDA");
    TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && a.size(1) == b.size(1) && a.is_contiguous() && b.is_contiguous(),
                "gemm_mxfp8: A [M, K], B [N, K] contiguous");
    const int64_t M = a.size(0), N = b.size(0), K = a.size(1);
    TORCH_CHECK(sfa.numel() >= (M + 127) / 128 * 128 * K / 32 && sfb.numel() >= (N + 127) / 128 * 128 * K / 32,
                "gemm_mxfp8: scale records too small");
    c10::cuda::CUDAGuard g(a.device());
    auto d = torch::empty({M, N}, a.options().dtype(at::kBFloat16));
    ttb::gemm_mxfp8(a.data_ptr(), b.data_ptr(), sfa.data_ptr(), sfb.data_ptr(), d.data_ptr(), M, N, K, stream(),
                    static_cast<int>(tile_n));
    return d;
  }, py::arg("a"), py::arg("sfa"), py::arg("b"), py::arg("sfb"), py::arg("tile_n") = 0);
  m.def("gemm_mxfp8_grouped", [](Tensor a, Tensor sfa, Tensor b, Tensor sfb, Tensor tile_group, int64_t n,
                                 int64_t tile_n) {
    // a [P, K] rows padded per group to 128; b [G*n, K] stacked groups; tile_group [P/128] int32
    TORCH_CHECK(a.is_cuda() && b.is_cuda() && a.scalar_type() == at::kByte && b.scalar_type() == at::kByte,
                "gemm_mxfp8_grouped: uint8 FP8 codes on CUDA");
    TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && a.size(1) == b.size(1) && a.is_contiguous() && b.is_contiguous(),
                "gemm_mxfp8_grouped: A [P, K], B [G*N, K] contiguous");
    const int64_t M = a.size(0), K = a.size(1);
    TORCH_CHECK(n > 0 && n % 128 == 0 && b.size(0) % n == 0, "gemm_mxfp8_grouped: N per group a multiple of 128");
    TORCH_CHECK(M % 128 == 0, "gemm_mxfp8_grouped: rows padded to 128");
    TORCH_CHECK(tile_group.is_cuda() && tile_group.scalar_type() == at::kInt && tile_group.is_contiguous() &&
                    tile_group.numel() == M / 128, "gemm_mxfp8_grouped: tile_group int32 [P/128]");
    const int64_t G = b.size(0) / n;
    TORCH_CHECK(sfa.numel() >= M * K / 32 && sfb.numel() >= G * n * K / 32, "gemm_mxfp8_grouped: scale records too small");
    c10::cuda::CUDAGuard g(a.device());
    auto d = torch::empty({M, n}, a.options().dtype(at::kBFloat16));
    ttb::MxEpilogue ep;
    ep.tile_group = tile_group.data_ptr<int>();
    ep.num_groups = static_cast<int>(G);
    ttb::gemm_mxfp8(a.data_ptr(), b.data_ptr(), sfa.data_ptr(), sfb.data_ptr(), d.data_ptr(), M, n, K, stream(),
                    static_cast<int>(tile_n), ep);
    return d;
  }, py::arg("a"), py::arg("sfa"), py::arg("b"), py::arg("sfb"), py::arg("tile_group"), py::arg("n"),
     py::arg("tile_n") = 0);
  m.def("moe_combine_fwd", [](c10::optional<Tensor> base, Tensor y, Tensor pos, c10::optional<Tensor> w) {
    // out[t] = base[t] + sum_j w[t, j] * y[pos[t, j]]: y [R, D] bf16, pos [T, k] int64, w [T, k] fp32
    check_cuda_bf16(y, "y");
    TORCH_CHECK(y.dim() == 2 && y.is_contiguous(), "moe_combine: y [R, D] contiguous");
    TORCH_CHECK(pos.is_cuda() && pos.scalar_type() == at::kLong && pos.dim() == 2 && pos.is_contiguous(),
                "moe_combine: pos [T, k] int64");
    const int64_t T = pos.size(0), k = pos.size(1), D = y.size(1);
    if (base.has_value()) {
      check_cuda_bf16(*base, "base");
      TORCH_CHECK(base->is_contiguous() && base->size(0) == T && base->size(1) == D, "moe_combine: base [T, D]");
    }
    if (w.has_value())
      TORCH_CHECK(w->is_cuda() && w->scalar_type() == at::kFloat && w->is_contiguous() && w->numel() == T * k,
                  "moe_combine: w [T, k] fp32");
    c10::cuda::CUDAGuard g(y.device());
    auto out = torch::empty({T, D}, y.options());
    ttb::moe_combine_fwd(base.has_value() ? base->data_ptr() : nullptr, y.data_ptr(), pos.data_ptr<int64_t>(),
                         w.has_value() ? w->data_ptr<float>() : nullptr, out.data_ptr(), T, (int)k, D, y.size(0),
                         stream());
    return out;
  });
  m.def("moe_combine_bwd", [](Tensor dout, Tensor y, Tensor pos, Tensor token_of, c10::optional<Tensor> scale,
                              bool need_dw) {
    // dy [R, D] = scale[r] * dout[token_of[r]]; dw [T, k] = dot(dout[t], y[pos[t, j]]) if need_dw
    check_cuda_bf16(dout, "dout");
    check_cuda_bf16(y, "y");
    TORCH_CHECK(dout.is_contiguous() && y.is_contiguous() && dout.size(1) == y.size(1), "moe_combine_bwd: rows");
    TORCH_CHECK(pos.scalar_type() == at::kLong && pos.is_contiguous() && token_of.scalar_type() == at::kLong &&
                    token_of.is_contiguous() && token_of.numel() == y.size(0), "moe_combine_bwd: indices");
    if (scale.has_value())
      TORCH_CHECK(scale->scalar_type() == at::kFloat && scale->is_contiguous() && scale->numel() == y.size(0),
                  "moe_combine_bwd: scale [R] fp32");
    const int64_t T = pos.size(0), k = pos.size(1), D = y.size(1), R = y.size(0);
    TORCH_CHECK(dout.size(0) == T, "moe_combine_bwd: dout [T, D]");
    c10::cuda::CUDAGuard g(y.device());
    auto dy = torch::empty({R, D}, y.options());
    auto dw = torch::empty({need_dw ? T : 0, need_dw ? k : 0}, y.options().dtype(at::kFloat));
    ttb::moe_combine_bwd(dout.data_ptr(), y.data_ptr(), pos.data_ptr<int64_t>(), token_of.data_ptr<int64_t>(),
                         scale.has_value() ? scale->data_ptr<float>() : nullptr, dy.data_ptr(),
                         need_dw ? dw.data_ptr<float>() : nullptr, T, (int)k, D, R, stream());
    return std::vector<Tensor>{dy, dw};
  });
  m.def("f8_quantize", [](Tensor x, bool rowwise) {
    check_cuda_bf16(x, "x");
    TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1, "f8_quantize: [R, C] with contiguous rows");
    c10::cuda::CUDAGuard g(x.device());
    const int64_t R = x.size(0), C = x.size(1), Cp = (C + 127) / 128 * 128;
    auto codes = torch::empty({R, Cp}, x.options().dtype(at::kByte));
    auto inv = torch::empty({rowwise ? R : 1}, x.options().dtype(at::kFloat));
    auto word = torch::empty({1}, x.options().dtype(at::kInt));
    ttb::f8_quantize(x.data_ptr(), R, C, x.stride(0), rowwise, codes.data_ptr(), inv.data_ptr<float>(),
                     reinterpret_cast<unsigned int*>(word.data_ptr<int>()), stream());
    return std::vector<Tensor>{codes, inv};
  });
  m.def("gemm_f8", [](Tensor a, Tensor a_inv, Tensor b, Tensor b_inv, int64_t tile_n) {
    TORCH_CHECK(a.is_cuda() && b.is_cuda() && a.scalar_type() == at::kByte && b.scalar_type() == at::kByte,
                "gemm_f8: uint8 E4M3 codes on CUDA");
    TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && a.size(1) == b.size(1) && a.is_contiguous() && b.is_contiguous(),
                "gemm_f8: A [M, K], B [N, K] contiguous");
    const int64_t M = a.size(0), N = b.size(0), K = a.size(1);
    TORCH_CHECK(a_inv.scalar_type() == at::kFloat && b_inv.scalar_type() == at::kFloat && a_inv.is_contiguous() &&
                    b_inv.is_contiguous() && (a_inv.numel() == M || a_inv.numel() == 1) &&
                    (b_inv.numel() == N || b_inv.numel() == 1),
                "gemm_f8: fp32 inverse scales, one per row or one per operand");
    c10::cuda::CUDAGuard g(a.device());
    auto d = torch::empty({M, N}, a.options().dtype(at::kBFloat16));
    ttb::MxEpilogue ep;
    ep.sa = a_inv.data_ptr<float>();
    ep.sb = b_inv.data_ptr<float>();
    ep.sa_rows = a_inv.numel() == M && M > 1;
    ep.sb_rows = b_inv.numel() == N && N > 1;
    ttb::gemm_mxfp8(a.data_ptr(), b.data_ptr(), nullptr, nullptr, d.data_ptr(), M, N, K, stream(),
                    static_cast<int>(tile_n), ep);
    return d;
  }, py::arg("a"), py::arg("a_inv"), py::arg("b"), py::arg("b_inv"), py::arg("tile_n") = 0);
  m.def("kda_gram_fwd", [](Tensor a, Tensor b, Tensor G, bool strict) {
    for (const Tensor* t : {&a, &b, &G})
      TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kFloat && t->is_contiguous() && t->dim() == 3 &&
                      t->sizes() == a.sizes(), "kda_gram: a, b, G contiguous fp32 [N, C, K]");
    c10::cuda::CUDAGuard g(a.device());
    auto out = torch::empty({a.size(0), a.size(1), a.size(1)}, a.options());
    ttb::kda_gram_fwd(a.data_ptr<float>(), b.data_ptr<float>(), G.data_ptr<float>(), out.data_ptr<float>(),
                      a.size(0), (int)a.size(1), (int)a.size(2), strict, stream());
    return out;
  });
  m.def("kda_gram_bwd", [](Tensor dout, Tensor a, Tensor b, Tensor G, bool strict) {
    TORCH_CHECK(dout.is_cuda() && dout.scalar_type() == at::kFloat && dout.is_contiguous(), "kda_gram: dout");
    c10::cuda::CUDAGuard g(a.device());
    auto da = torch::empty_like(a), db = torch::empty_like(b), dG = torch::empty_like(G);
    ttb::kda_gram_bwd(dout.data_ptr<float>(), a.data_ptr<float>(), b.data_ptr<float>(), G.data_ptr<float>(),
                      da.data_ptr<float>(), db.data_ptr<float>(), dG.data_ptr<float>(), a.size(0), (int)a.size(1),
                      (int)a.size(2), strict, stream());
    return std::vector<Tensor>{da, db, dG};
  });
  // chunked-KDA state recurrence on tcgen05 (C = 64, K = V = 128): bf16 w / kdec [BH,NT,C,K],
  // u^T [BH,NT,V,C]; fp32 dec [BH,NT,K], optional S0^T [BH,V,K].
  // Returns states^T [BH,NT,V,K] bf16 (state at each chunk start), v'^T [BH,NT,V,C] bf16, final S^T fp32.
  m.def("kda_prep_fwd", [](Tensor q, Tensor k, Tensor g, int64_t C) {
    for (const Tensor* t : {&q, &k, &g})
      TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kFloat && t->is_contiguous() && t->dim() == 4 &&
                      t->sizes() == q.sizes(),
                  "kda_prep_fwd: q, k, g fp32 contiguous [B, T, H, K] of one shape");
    c10::cuda::CUDAGuard guard(q.device());
    const int64_t B = q.size(0), T = q.size(1), H = q.size(2), K = q.size(3), NT = (T + C - 1) / C;
    auto o = q.options();
    auto qc = torch::empty({B * H, NT, C, K}, o), kc = torch::empty_like(qc), G = torch::empty_like(qc);
    auto kg = torch::empty_like(qc), qg = torch::empty_like(qc), kd = torch::empty_like(qc);
    auto decay = torch::empty({B * H, NT, K}, o);
    ttb::kda_prep_fwd(q.data_ptr<float>(), k.data_ptr<float>(), g.data_ptr<float>(), (int)B, (int)T, (int)H, (int)K,
                      (int)C, qc.data_ptr<float>(), kc.data_ptr<float>(), G.data_ptr<float>(), kg.data_ptr<float>(),
                      qg.data_ptr<float>(), kd.data_ptr<float>(), decay.data_ptr<float>(), stream());
    return std::vector<Tensor>{qc, kc, G, kg, qg, kd, decay};
  });
  m.def("kda_prep_bwd", [](Tensor q, Tensor k, Tensor G, int64_t C, c10::optional<Tensor> dqc,
                           c10::optional<Tensor> dkc, c10::optional<Tensor> dG, c10::optional<Tensor> dkg,
                           c10::optional<Tensor> dqg, c10::optional<Tensor> dkd, c10::optional<Tensor> ddecay) {
    c10::cuda::CUDAGuard guard(q.device());
    auto ptr = [&](const c10::optional<Tensor>& t, const char* name) -> const float* {
      if (!t.has_value() || !t->defined()) return nullptr;
      TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kFloat && t->is_contiguous(), "kda_prep_bwd: ", name,
                  " must be fp32 contiguous");
      return t->data_ptr<float>();
    };
    const int64_t B = q.size(0), T = q.size(1), H = q.size(2), K = q.size(3);
    auto dq = torch::empty_like(q), dk = torch::empty_like(q), dg = torch::empty_like(q);
    ttb::kda_prep_bwd(q.data_ptr<float>(), k.data_ptr<float>(), G.data_ptr<float>(), (int)B, (int)T, (int)H, (int)K,
                      (int)C, ptr(dqc, "dqc"), ptr(dkc, "dkc"), ptr(dG, "dG"), ptr(dkg, "dkg"), ptr(dqg, "dqg"),
                      ptr(dkd, "dkd"), ptr(ddecay, "ddecay"), dq.data_ptr<float>(), dk.data_ptr<float>(),
                      dg.data_ptr<float>(), stream());
    return std::vector<Tensor>{dq, dk, dg};
  });
  m.def("kda_state_fwd", [](Tensor w, Tensor kd, Tensor uT, Tensor dec, c10::optional<Tensor> S0) {
    for (const Tensor* t : {&w, &kd, &uT})
      TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kBFloat16 && t->is_contiguous(), "kda_state: bf16");
    TORCH_CHECK(dec.is_cuda() && dec.scalar_type() == at::kFloat && dec.is_contiguous(), "kda_state: dec fp32");
    const int64_t BH = w.size(0), NT = w.size(1);
    TORCH_CHECK(w.dim() == 4 && w.size(2) == 64 && w.size(3) == 128 && kd.sizes() == w.sizes() &&
                    uT.sizes() == at::IntArrayRef({BH, NT, 128, 64}) && dec.sizes() == at::IntArrayRef({BH, NT, 128}),
                "kda_state: shapes (C = 64, K = V = 128)");
    if (S0.has_value())
      TORCH_CHECK(S0->is_cuda() && S0->scalar_type() == at::kFloat && S0->is_contiguous() &&
                      S0->sizes() == at::IntArrayRef({BH, 128, 128}), "kda_state: S0 fp32 [BH, V, K]");
    c10::cuda::CUDAGuard g(w.device());
    auto states = torch::empty({BH, NT, 128, 128}, w.options());
    auto vnT = torch::empty({BH, NT, 128, 64}, w.options());
    auto fin = torch::empty({BH, 128, 128}, dec.options());
    ttb::kda_state_fwd(w.data_ptr(), kd.data_ptr(), uT.data_ptr(), dec.data_ptr<float>(),
                       S0.has_value() ? S0->data_ptr<float>() : nullptr, states.data_ptr(), vnT.data_ptr(),
                       fin.data_ptr<float>(), (int)BH, (int)NT, stream());
    return std::vector<Tensor>{states, vnT, fin};
  });
  // backward: bf16 qg / w / kdec [BH,NT,C,K], dO [BH,NT,C,V], Aqk [BH,NT,C,C]; fp32 dec, optional dSfin^T.
  // Returns dstates^T [BH,NT,V,K] bf16 (gradient of the state after each chunk), dv'^T fp32, dS0^T fp32.
  m.def("kda_state_bwd", [](Tensor qg, Tensor w, Tensor kd, Tensor dO, Tensor Aqk, Tensor dec,
                            c10::optional<Tensor> dSfin) {
    for (const Tensor* t : {&qg, &w, &kd, &dO, &Aqk})
      TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kBFloat16 && t->is_contiguous(), "kda_state: bf16");
    const int64_t BH = w.size(0), NT = w.size(1);
    TORCH_CHECK(w.dim() == 4 && w.size(2) == 64 && w.size(3) == 128 && qg.sizes() == w.sizes() &&
                    kd.sizes() == w.sizes() && dO.sizes() == at::IntArrayRef({BH, NT, 64, 128}) &&
                    Aqk.sizes() == at::IntArrayRef({BH, NT, 64, 64}) && dec.sizes() == at::IntArrayRef({BH, NT, 128}),
                "kda_state_bwd: shapes (C = 64, K = V = 128)");
    TORCH_CHECK(dec.is_cuda() && dec.scalar_type() == at::kFloat && dec.is_contiguous(), "kda_state: dec fp32");
    if (dSfin.has_value())
      TORCH_CHECK(dSfin->is_cuda() && dSfin->scalar_type() == at::kFloat && dSfin->is_contiguous() &&
                      dSfin->sizes() == at::IntArrayRef({BH, 128, 128}), "kda_state: dSfin fp32 [BH, V, K]");
    c10::cuda::CUDAGuard g(w.device());
    auto dstates = torch::empty({BH, NT, 128, 128}, w.options());
    auto duT = torch::empty({BH, NT, 128, 64}, dec.options());
    auto dS0 = torch::empty({BH, 128, 128}, dec.options());
    ttb::kda_state_bwd(qg.data_ptr(), w.data_ptr(), kd.data_ptr(), dO.data_ptr(), Aqk.data_ptr(),
                       dec.data_ptr<float>(), dSfin.has_value() ? dSfin->data_ptr<float>() : nullptr,
                       dstates.data_ptr(), duT.data_ptr<float>(), dS0.data_ptr<float>(), (int)BH, (int)NT, stream());
    return std::vector<Tensor>{dstates, duT, dS0};
  });
  m.def("kda_state_error_code", &ttb::kda_state_error_code, py::arg("reset") = true);
  // chunked-KDA inter-chunk recurrence: u [BH,NT,C,V], w/qg/kdec [BH,NT,C,K], Aqk [BH,NT,C,C], dec [BH,NT,K]
  m.def("kda_scan_fwd", [](Tensor u, Tensor w, Tensor qg, Tensor Aqk, Tensor kdec, Tensor dec, int64_t vs) {
    for (const Tensor* t : {&u, &w, &qg, &Aqk, &kdec, &dec})
      TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kFloat && t->is_contiguous(), "kda_scan: contiguous fp32");
    TORCH_CHECK(u.dim() == 4 && w.dim() == 4 && Aqk.dim() == 4 && dec.dim() == 3, "kda_scan: ranks");
    const int64_t BH = u.size(0), NT = u.size(1), C = u.size(2), V = u.size(3), K = w.size(3);
    TORCH_CHECK(w.sizes() == qg.sizes() && w.sizes() == kdec.sizes() && w.size(0) == BH && w.size(1) == NT &&
                    w.size(2) == C && Aqk.size(2) == C && Aqk.size(3) == C && dec.size(2) == K,
                "kda_scan: shapes");
    c10::cuda::CUDAGuard g(u.device());
    auto o = torch::empty_like(u);
    auto states = torch::empty({BH, NT, K, V}, u.options());
    auto fin = torch::empty({BH, K, V}, u.options());
    ttb::kda_scan_fwd(u.data_ptr<float>(), w.data_ptr<float>(), qg.data_ptr<float>(), Aqk.data_ptr<float>(),
                      kdec.data_ptr<float>(), dec.data_ptr<float>(), o.data_ptr<float>(), states.data_ptr<float>(),
                      fin.data_ptr<float>(), BH, (int)NT, (int)C, (int)K, (int)V, (int)vs, stream());
    return std::vector<Tensor>{o, states, fin};
  });
  m.def("kda_scan_bwd", [](Tensor dO, Tensor u, Tensor w, Tensor qg, Tensor Aqk, Tensor kdec, Tensor dec,
                           Tensor states, int64_t vs) {
    TORCH_CHECK(dO.is_cuda() && dO.scalar_type() == at::kFloat && dO.is_contiguous() && dO.sizes() == u.sizes(),
                "kda_scan: dO");
    const int64_t BH = u.size(0), NT = u.size(1), C = u.size(2), V = u.size(3), K = w.size(3);
    TORCH_CHECK(V % vs == 0, "kda_scan: V must be a multiple of the slice width");
    const int64_t ns = V / vs;
    c10::cuda::CUDAGuard g(u.device());
    auto du = torch::empty_like(u);
    auto dqg = torch::empty({ns, BH, NT, C, K}, u.options()), dw = torch::empty_like(dqg),
         dkd = torch::empty_like(dqg);
    auto dA = torch::empty({ns, BH, NT, C, C}, u.options());
    auto dd = torch::empty({ns, BH, NT, K}, u.options());
    ttb::kda_scan_bwd(dO.data_ptr<float>(), u.data_ptr<float>(), w.data_ptr<float>(), qg.data_ptr<float>(),
                      Aqk.data_ptr<float>(), kdec.data_ptr<float>(), dec.data_ptr<float>(), states.data_ptr<float>(),
                      du.data_ptr<float>(), dqg.data_ptr<float>(), dw.data_ptr<float>(), dkd.data_ptr<float>(),
                      dA.data_ptr<float>(), dd.data_ptr<float>(), BH, (int)NT, (int)C, (int)K, (int)V, (int)vs,
                      stream());
    return std::vector<Tensor>{du, dqg.sum(0), dw.sum(0), dkd.sum(0), dA.sum(0), dd.sum(0)};
  });
  m.def("router_topk", [](Tensor logits, c10::optional<Tensor> bias, int64_t top_k, bool sigmoid, int64_t n_groups,
                          int64_t n_limited) {
    TORCH_CHECK(logits.is_cuda() && logits.scalar_type() == at::kFloat && logits.is_contiguous() && logits.dim() == 2,
                "router_topk: logits contiguous fp32 [T, E]");
    const int64_t T = logits.size(0), E = logits.size(1);
    const float* b = nullptr;
    Tensor bc;
    if (bias.has_value()) {
      bc = bias->to(at::kFloat).contiguous();
      TORCH_CHECK(bc.is_cuda() && bc.numel() == E, "router_topk: bias [E]");
      b = bc.data_ptr<float>();
    }
    c10::cuda::CUDAGuard g(logits.device());
    auto idx = torch::empty({T, top_k}, logits.options().dtype(at::kLong));
    auto counts = torch::empty({E}, logits.options().dtype(at::kInt));
    ttb::router_topk(logits.data_ptr<float>(), b, T, (int)E, (int)top_k, sigmoid, (int)n_groups, (int)n_limited,
                     idx.data_ptr<int64_t>(), counts.data_ptr<int32_t>(), stream());
    return std::vector<Tensor>{idx, counts};
  });
  // block attention residuals: blocks = completed blocks + partial, each contiguous bf16 [T, D]
  m.def("attn_res_fwd", [](std::vector<Tensor> blocks, Tensor u, double eps) {
    TORCH_CHECK(!blocks.empty() && u.is_cuda() && u.scalar_type() == at::kFloat && u.is_contiguous(), "attn_res: u");
    const int64_t D = u.numel(), T = blocks[0].numel() / D;
    std::vector<const void*> ptrs;
    for (auto& b : blocks) {
      TORCH_CHECK(b.is_cuda() && b.scalar_type() == at::kBFloat16 && b.is_contiguous() && b.numel() == T * D,
                  "attn_res: blocks contiguous bf16 of one shape");
      ptrs.push_back(b.data_ptr());
    }
    c10::cuda::CUDAGuard g(u.device());
    auto out = torch::empty_like(blocks[0]);
    ttb::attn_res_fwd(ptrs.data(), (int)ptrs.size(), u.data_ptr<float>(), out.data_ptr(), T, (int)D, (float)eps,
                      stream());
    return out;
  });
  m.def("attn_res_bwd", [](std::vector<Tensor> blocks, Tensor u, Tensor dout, double eps) {
    const int64_t D = u.numel(), T = blocks[0].numel() / D;
    TORCH_CHECK(dout.is_cuda() && dout.scalar_type() == at::kBFloat16 && dout.is_contiguous() &&
                    dout.numel() == T * D, "attn_res: dout");
    std::vector<const void*> ptrs;
    std::vector<void*> dptrs;
    std::vector<Tensor> grads;
    for (auto& b : blocks) {
      ptrs.push_back(b.data_ptr());
      grads.push_back(torch::empty_like(b));
      dptrs.push_back(grads.back().data_ptr());
    }
    c10::cuda::CUDAGuard g(u.device());
    auto du = torch::empty_like(u);
    ttb::attn_res_bwd(ptrs.data(), dptrs.data(), (int)ptrs.size(), u.data_ptr<float>(), dout.data_ptr(),
                      du.data_ptr<float>(), T, (int)D, (float)eps, stream());
    grads.push_back(du);
    return grads;
  });
  m.def("kda_short_conv_fwd", [](Tensor x, Tensor w) {  // x [B, T, C] bf16, w [C, W] fp32
    TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.is_contiguous() && x.dim() == 3, "short conv: x");
    TORCH_CHECK(w.scalar_type() == at::kFloat && w.is_contiguous() && w.size(0) == x.size(2), "short conv: w");
    c10::cuda::CUDAGuard g(x.device());
    auto y = torch::empty_like(x);
    ttb::kda_short_conv_fwd(x.data_ptr(), w.data_ptr<float>(), y.data_ptr(), x.size(0), x.size(1), (int)x.size(2),
                            (int)w.size(1), stream());
    return y;
  });
  m.def("kda_short_conv_bwd", [](Tensor x, Tensor w, Tensor dy) {
    TORCH_CHECK(dy.sizes() == x.sizes() && dy.is_contiguous() && dy.scalar_type() == at::kBFloat16, "short conv: dy");
    c10::cuda::CUDAGuard g(x.device());
    auto dx = torch::empty_like(x);
    auto dw = torch::empty_like(w);
    ttb::kda_short_conv_bwd(x.data_ptr(), w.data_ptr<float>(), dy.data_ptr(), dx.data_ptr(), dw.data_ptr<float>(),
                            x.size(0), x.size(1), (int)x.size(2), (int)w.size(1), stream());
    return std::vector<Tensor>{dx, dw};
  });
  m.def("kda_gated_norm_fwd", [](Tensor x, Tensor z, Tensor gw, double eps) {  // rows of width D = gw.numel()
    TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.is_contiguous() && z.sizes() == x.sizes() &&
                    z.scalar_type() == at::kBFloat16 && z.is_contiguous(), "gated norm: x, z");
    TORCH_CHECK(gw.scalar_type() == at::kFloat && gw.is_contiguous() && x.size(-1) == gw.numel(), "gated norm: g");
    c10::cuda::CUDAGuard g(x.device());
    auto y = torch::empty_like(x);
    ttb::kda_gated_norm_fwd(x.data_ptr(), z.data_ptr(), gw.data_ptr<float>(), y.data_ptr(), x.numel() / gw.numel(),
                            (int)gw.numel(), (float)eps, stream());
    return y;
  });
  m.def("kda_gated_norm_bwd", [](Tensor x, Tensor z, Tensor gw, Tensor dy, double eps) {
    TORCH_CHECK(dy.sizes() == x.sizes() && dy.is_contiguous() && dy.scalar_type() == at::kBFloat16, "gated norm: dy");
    c10::cuda::CUDAGuard g(x.device());
    auto dx = torch::empty_like(x), dz = torch::empty_like(z), dg = torch::empty_like(gw);
    ttb::kda_gated_norm_bwd(x.data_ptr(), z.data_ptr(), gw.data_ptr<float>(), dy.data_ptr(), dx.data_ptr(),
                            dz.data_ptr(), dg.data_ptr<float>(), x.numel() / gw.numel(), (int)gw.numel(), (float)eps,
                            stream());
    return std::vector<Tensor>{dx, dz, dg};
  });
  m.def("kda_gate_fwd", [](Tensor x, Tensor A, c10::optional<Tensor> b) {  // x [..., H, K] bf16, A [H], b [H*K]
    TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.is_contiguous() && x.dim() >= 2, "kda gate: x");
    const int64_t H = x.size(-2), K = x.size(-1);
    TORCH_CHECK(A.scalar_type() == at::kFloat && A.is_contiguous() && A.numel() == H, "kda gate: A");
    const float* bp = nullptr;
    if (b.has_value()) {
      TORCH_CHECK(b->scalar_type() == at::kFloat && b->is_contiguous() && b->numel() == H * K, "kda gate: bias");
      bp = b->data_ptr<float>();
    }
    c10::cuda::CUDAGuard g(x.device());
    auto out = torch::empty(x.sizes(), x.options().dtype(at::kFloat));
    ttb::kda_gate_fwd(x.data_ptr(), A.data_ptr<float>(), bp, out.data_ptr<float>(), x.numel(), (int)H, (int)K,
                      stream());
    return out;
  });
  m.def("kda_gate_bwd", [](Tensor x, Tensor A, c10::optional<Tensor> b, Tensor dg) {
    TORCH_CHECK(dg.scalar_type() == at::kFloat && dg.is_contiguous() && dg.sizes() == x.sizes(), "kda gate: dg");
    const int64_t H = x.size(-2), K = x.size(-1);
    c10::cuda::CUDAGuard g(x.device());
    auto dx = torch::empty_like(x);
    auto dA = torch::empty_like(A);
    Tensor db = b.has_value() ? torch::empty_like(*b) : Tensor();
    ttb::kda_gate_bwd(x.data_ptr(), A.data_ptr<float>(), b.has_value() ? b->data_ptr<float>() : nullptr,
                      dg.data_ptr<float>(), dx.data_ptr(), dA.data_ptr<float>(),
                      b.has_value() ? db.data_ptr<float>() : nullptr, x.numel(), (int)H, (int)K, stream());
    return std::vector<Tensor>{dx, dA, b.has_value() ? db : torch::zeros({0}, A.options())};
  });
  m.def("mxgemm_error_code", &ttb::mxgemm_error_code, py::arg("reset") = true);
  m.def("dp_error_info", []() {
    int v[4];
    ttb::dp_error_info(v);
    return std::vector<int>(v, v + 4);
  });
  m.def("multi_sumsq", &multi_sumsq, "sum of squares over a list of fp32/bf16 tensors");
  m.def("multi_clip_scale", &multi_clip_scale, "scale tensors by min(1, max_norm/(sqrt(total)+1e-6))");
  m.def("attn_fwd", &attn_fwd, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("causal"), py::arg("scale"),
        py::arg("doc_start") = py::none(), py::arg("doc_end") = py::none());
  m.def("attn_bwd", &attn_bwd, py::arg("dout"), py::arg("q"), py::arg("k"), py::arg("v"), py::arg("o"),
        py::arg("lse"), py::arg("causal"), py::arg("scale"), py::arg("dlse") = py::none(),
        py::arg("doc_start") = py::none(), py::arg("doc_end") = py::none());
}
