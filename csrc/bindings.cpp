// Python bindings of the sm_100a kernels: tensor validation, output allocation and stream
// selection.  This is the only translation unit that includes torch headers.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "launchers.h"

namespace pan {

const char* launch_qkv_post_fwd(const void* raw, const float* qw, const float* kw, const float* cos_t,
                                const float* sin_t, const int* itc, int nv, int na, int L, int H, int D, float eps,
                                void* q, void* k, void* v, cudaStream_t s, const uint64_t* peer_q = nullptr,
                                const uint64_t* peer_k = nullptr, const uint64_t* peer_v = nullptr, int cp = 1,
                                int rank = 0);
const char* launch_qkv_post_bwd(const void* dq, const void* dk, const void* dv, const void* raw, const float* qw,
                                const float* kw, const float* cos_t, const float* sin_t, const int* itc, int nv,
                                int na, int L, int H, int D, float eps, void* draw, float* dqw, float* dkw,
                                cudaStream_t s);

const char* launch_attn_fwd(const void* q, const void* k, const void* v, const int* items, int n_items, int L, int H,
                            int head_dim, float scale, void* out, float* lse, cudaStream_t s,
                            const uint64_t* o_peer = nullptr, int cp = 1, int head_base = 0, int H_total = 0);
const char* launch_attn_bwd_cp(const void* q, const void* k, const void* v, const void* o, const float* lse,
                               const int* items_kv, int n_items_kv, int L, int H, int head_dim, float scale,
                               int n_valid, float* delta, void* dout_head, float* dq_acc, const uint64_t* do_peer,
                               const uint64_t* dq_peer, const uint64_t* dk_peer, const uint64_t* dv_peer, int cp,
                               int head_base, int H_total, cudaStream_t s);
const char* launch_attn_bwd(const void* q, const void* k, const void* v, const void* o, const void* dout,
                            const float* lse, const int* items_q, int n_items_q, const int* items_kv, int n_items_kv,
                            int L, int H, int head_dim, float scale, float* delta, void* dq, void* dk, void* dv,
                            float* dq_acc, cudaStream_t s);
int attn_error_flag(bool reset);
int qkv_bounds_error(bool reset);
void attn_set_forward_variant(int v);
int attn_get_variant(int backward);
void launch_sumsq(const void* x, bool fp32, size_t n, float* partial, int n_part, cudaStream_t s);
void launch_reduce_clip(const float* partial, int n, float max_norm, float* out, cudaStream_t s);
void launch_muon_momentum(float* buf, const void* g, bool g_fp32, const float* clip, float mu, size_t n, void* u,
                          cudaStream_t s);
void launch_muon_update(void* hi, void* lo, const void* u, const float* lr, float lr_scale, float wd, size_t n,
                        cudaStream_t s);
void launch_adamw_update(void* hi, void* lo, const void* g, bool g_fp32, float* m, float* v, const float* clip,
                         const float* lr, float beta1, float beta2, float eps, float wd, float bc1, float bc2_sqrt,
                         size_t n, cudaStream_t s);
void launch_split_master(const float* x, void* hi, void* lo, size_t n, cudaStream_t s);
void launch_join_master(const void* hi, const void* lo, float* x, size_t n, cudaStream_t s);
void launch_trace(const float* R, int batch, int M, float* out, cudaStream_t s);
void launch_gram_normalize(const float* R, const float* norm2, int batch, int M, float eps, void* Rn, cudaStream_t s);
void launch_add_diag(void* Z, int batch, int M, float a, cudaStream_t s);
void launch_scale_by_invnorm(void* Q, const float* norm2, int batch, int M, float eps, cudaStream_t s);

namespace {

cudaStream_t stream() { return at::cuda::getCurrentCUDAStream(); }

void check_launch(const char* err, const char* what) {
  TORCH_CHECK(err == nullptr, what, ": ", err ? err : "");
  cudaError_t e = cudaGetLastError();
  TORCH_CHECK(e == cudaSuccess, what, ": ", cudaGetErrorString(e));
}

void check_rows(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == torch::kBFloat16 && t.dim() == 2 && t.is_contiguous(), name,
              " must be a contiguous bf16 CUDA [L, C] tensor");
  TORCH_CHECK(t.size(1) % 256 == 0, name, ": C must be a multiple of 256");
}

void check_bf16(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == torch::kBFloat16 && t.is_contiguous(), name,
              " must be a contiguous bf16 CUDA tensor");
}

void check_i32(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == torch::kInt32 && t.is_contiguous(), name,
              " must be a contiguous int32 CUDA tensor");
}

}  // namespace

// ------------------------------------------------------------------ packed elementwise ops
torch::Tensor ln_modulate_fwd(torch::Tensor x, torch::Tensor stats, torch::Tensor shift, torch::Tensor scale,
                              torch::Tensor bounds, int64_t n_seg) {
  const at::cuda::CUDAGuard guard(x.device());
  check_rows(x, "x");
  check_bf16(shift, "shift");
  check_bf16(scale, "scale");
  check_i32(bounds, "bounds");
  TORCH_CHECK(stats.scalar_type() == torch::kFloat32 && stats.is_contiguous(), "stats must be fp32 [L, 2]");
  TORCH_CHECK(n_seg <= 64 && shift.size(0) >= n_seg && scale.size(0) >= n_seg, "bad segment count");
  auto y = torch::empty_like(x);
  launch_ln_modulate_fwd(x.data_ptr(), stats.data_ptr<float>(), shift.data_ptr(), scale.data_ptr(),
                         bounds.data_ptr<int>(), n_seg, x.size(0), x.size(1), y.data_ptr(), stream());
  check_launch(nullptr, "ln_modulate_fwd");
  return y;
}

std::vector<torch::Tensor> ln_modulate_bwd(torch::Tensor g, torch::Tensor x, torch::Tensor stats, torch::Tensor scale,
                                           torch::Tensor bounds, int64_t n_seg) {
  const at::cuda::CUDAGuard guard(x.device());
  check_rows(g, "grad");
  check_rows(x, "x");
  check_bf16(scale, "scale");
  auto dx = torch::empty_like(x);
  auto opts = x.options().dtype(torch::kFloat32);
  auto dshift = torch::zeros({scale.size(0), x.size(1)}, opts);
  auto dscale = torch::zeros({scale.size(0), x.size(1)}, opts);
  launch_ln_modulate_bwd(g.data_ptr(), x.data_ptr(), stats.data_ptr<float>(), scale.data_ptr(), bounds.data_ptr<int>(),
                         n_seg, x.size(0), x.size(1), dx.data_ptr(), dshift.data_ptr<float>(),
                         dscale.data_ptr<float>(), stream());
  check_launch(nullptr, "ln_modulate_bwd");
  return {dx, dshift, dscale};
}

std::vector<torch::Tensor> gate_residual_fwd(torch::Tensor y, torch::Tensor gate, torch::Tensor res,
                                             torch::Tensor bounds, int64_t n_seg) {
  const at::cuda::CUDAGuard guard(y.device());
  check_rows(y, "y");
  check_rows(res, "residual");
  check_bf16(gate, "gate");
  auto out = torch::empty_like(res);
  auto stats = torch::empty({y.size(0), 2}, y.options().dtype(torch::kFloat32));
  launch_gate_residual_fwd(y.data_ptr(), gate.data_ptr(), res.data_ptr(), bounds.data_ptr<int>(), n_seg, y.size(0),
                           y.size(1), out.data_ptr(), stats.data_ptr<float>(), stream());
  check_launch(nullptr, "gate_residual_fwd");
  return {out, stats};
}

std::vector<torch::Tensor> gate_bwd(torch::Tensor g, torch::Tensor y, torch::Tensor gate, torch::Tensor bounds,
                                    int64_t n_seg) {
  const at::cuda::CUDAGuard guard(g.device());
  check_rows(g, "grad");
  check_rows(y, "y");
  auto dy = torch::empty_like(g);
  auto dgate = torch::zeros({gate.size(0), g.size(1)}, g.options().dtype(torch::kFloat32));
  launch_gate_bwd(g.data_ptr(), y.data_ptr(), gate.data_ptr(), bounds.data_ptr<int>(), n_seg, g.size(0), g.size(1),
                  dy.data_ptr(), dgate.data_ptr<float>(), stream());
  check_launch(nullptr, "gate_bwd");
  return {dy, dgate};
}

std::vector<torch::Tensor> simple_concat_fwd(torch::Tensor vid, torch::Tensor txt, c10::optional<torch::Tensor> ttv,
                                             int64_t total) {
  const at::cuda::CUDAGuard guard(vid.device());
  check_rows(vid, "video");
  check_rows(txt, "text");
  const int nv = vid.size(0), nt = txt.size(0);
  TORCH_CHECK(total >= nv + nt, "total rows smaller than video + text");
  auto out = torch::empty({total, vid.size(1)}, vid.options());
  auto stats = torch::empty({total, 2}, vid.options().dtype(torch::kFloat32));
  const void* tp = ttv.has_value() ? ttv.value().data_ptr() : nullptr;
  launch_concat_fwd(vid.data_ptr(), txt.data_ptr(), tp, nv, nt, total, vid.size(1), out.data_ptr(),
                    stats.data_ptr<float>(), stream());
  check_launch(nullptr, "simple_concat_fwd");
  return {out, stats};
}

torch::Tensor segment_sum(torch::Tensor x, torch::Tensor bounds, int64_t n_seg) {
  const at::cuda::CUDAGuard guard(x.device());
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kBFloat16 && x.dim() == 2 && x.is_contiguous() &&
                  x.size(1) % 8 == 0,
              "segment_sum: x must be a contiguous bf16 [L, C] CUDA tensor with C % 8 == 0");
  check_i32(bounds, "bounds");
  auto out = torch::zeros({n_seg, x.size(1)}, x.options().dtype(torch::kFloat32));
  launch_segment_sum(x.data_ptr(), bounds.data_ptr<int>(), n_seg, x.size(0), x.size(1), out.data_ptr<float>(),
                     stream());
  check_launch(nullptr, "segment_sum");
  return out;
}

torch::Tensor column_sum(torch::Tensor x) {
  auto b = torch::tensor({0, (int)x.size(0)}, x.options().dtype(torch::kInt32));
  return segment_sum(x, b, 1)[0];
}

torch::Tensor mse_fwd(torch::Tensor pred, torch::Tensor tgt, int64_t nv) {
  const at::cuda::CUDAGuard guard(pred.device());
  check_bf16(pred, "pred");
  check_bf16(tgt, "target");
  TORCH_CHECK(pred.size(1) == tgt.size(1) && tgt.size(0) >= nv && pred.size(0) >= nv, "shape mismatch");
  const size_t n = (size_t)nv * pred.size(1);
  TORCH_CHECK(n % 8 == 0, "element count must be a multiple of 8");
  const int parts = 148 * 4;
  auto partial = torch::empty({parts}, pred.options().dtype(torch::kFloat32));
  auto out = torch::empty({2}, pred.options().dtype(torch::kFloat32));
  launch_mse_fwd(pred.data_ptr(), tgt.data_ptr(), n, partial.data_ptr<float>(), parts, out.data_ptr<float>(),
                 stream());
  check_launch(nullptr, "mse_fwd");
  return out;
}

torch::Tensor mse_bwd(torch::Tensor pred, torch::Tensor tgt, torch::Tensor gsum, int64_t nv) {
  const at::cuda::CUDAGuard guard(pred.device());
  auto dpred = torch::empty_like(pred);
  launch_mse_bwd(pred.data_ptr(), tgt.data_ptr(), gsum.data_ptr<float>(), (size_t)nv * pred.size(1), pred.numel(),
                 dpred.data_ptr(), stream());
  check_launch(nullptr, "mse_bwd");
  return dpred;
}

torch::Tensor gather_rows(torch::Tensor x, torch::Tensor idx) {
  const at::cuda::CUDAGuard guard(x.device());
  TORCH_CHECK(x.is_contiguous(), "gather_rows: x must be contiguous");
  check_i32(idx, "idx");
  const int rows = idx.size(0);
  const int64_t row_bytes = x.numel() / x.size(0) * x.element_size();
  TORCH_CHECK(row_bytes % 16 == 0, "row size must be a multiple of 16 bytes");
  std::vector<int64_t> shape(x.sizes().begin(), x.sizes().end());
  shape[0] = rows;
  auto out = torch::empty(shape, x.options());
  launch_gather_rows(x.data_ptr(), idx.data_ptr<int>(), rows, (int)(row_bytes / 16), out.data_ptr(), stream());
  check_launch(nullptr, "gather_rows");
  return out;
}

// ------------------------------------------------------------------ GEMM
namespace {

GemmArgs base_args(const torch::Tensor& A, bool a_kmajor, torch::Tensor& D) {

  TORCH_CHECK(A.is_cuda() && A.scalar_type() == torch::kBFloat16 && A.dim() == 2 && A.stride(1) == 1,
              "A must be a row-major bf16 CUDA matrix");
  TORCH_CHECK(D.is_cuda() && D.dim() == 2 && D.stride(1) == 1 &&
                  (D.scalar_type() == torch::kBFloat16 || D.scalar_type() == torch::kFloat32),
              "D must be a row-major bf16/fp32 CUDA matrix");
  GemmArgs a{};
  a.A = A.data_ptr();
  a.lda = A.stride(0);
  a.a_mn = a_kmajor ? 0 : 1;
  a.M = a_kmajor ? A.size(0) : A.size(1);
  a.K = a_kmajor ? A.size(1) : A.size(0);
  a.D = D.data_ptr();
  a.ldd = D.stride(0);
  a.d_fp32 = D.scalar_type() == torch::kFloat32;
  return a;
}

void set_group(GemmArgs& a, int g, const torch::Tensor& B, bool b_kmajor, int row_begin, int row_end,
               const c10::optional<torch::Tensor>& bias) {
  TORCH_CHECK(B.is_cuda() && B.scalar_type() == torch::kBFloat16 && B.dim() == 2 && B.stride(1) == 1,
              "B must be a row-major bf16 CUDA matrix");
  GemmGroup& gr = a.groups[g];
  gr.B = B.data_ptr();
  gr.ldb = B.stride(0);
  gr.n = b_kmajor ? B.size(0) : B.size(1);
  gr.k = b_kmajor ? B.size(1) : B.size(0);
  gr.row_begin = row_begin;
  gr.row_end = row_end;
  gr.bias = nullptr;
  if (bias.has_value()) {
    const auto& b = bias.value();
    TORCH_CHECK(b.scalar_type() == torch::kBFloat16 && b.is_contiguous() && b.numel() >= gr.n, "bias must be bf16 [N]");
    gr.bias = b.data_ptr();
  }
}

}  // namespace

void gemm(torch::Tensor A, torch::Tensor B, torch::Tensor D, bool a_kmajor, bool b_kmajor,
          c10::optional<torch::Tensor> bias, c10::optional<torch::Tensor> gelu_pre, bool accumulate) {
  const at::cuda::CUDAGuard guard(A.device());
  GemmArgs a = base_args(A, a_kmajor, D);
  a.b_mn = b_kmajor ? 0 : 1;
  a.n_groups = 1;
  set_group(a, 0, B, b_kmajor, 0, a.M, bias);
  TORCH_CHECK(a.groups[0].k == a.K, "K mismatch");
  TORCH_CHECK(D.size(0) >= a.M && D.size(1) >= a.groups[0].n, "D too small");
  if (gelu_pre.has_value()) {
    const auto& p = gelu_pre.value();
    TORCH_CHECK(p.scalar_type() == torch::kBFloat16 && p.stride(1) == 1, "gelu_pre must be bf16 row-major");
    a.epi = 1;
    a.aux = p.data_ptr();
    a.ldaux = p.stride(0);
  }
  a.accumulate = accumulate ? 1 : 0;
  check_launch(launch_gemm(a, stream()), "gemm");
}

// Batched D[b] = alpha * A[b] @ B[b]^T + beta * C[b] over 3-D tensors [batch, rows, cols] (row-major
// in the last two dims); operand majors as in gemm().  C may alias D.
void gemm_batched(torch::Tensor A, torch::Tensor B, torch::Tensor D, bool a_kmajor, bool b_kmajor, double alpha,
                  double beta, c10::optional<torch::Tensor> C) {
  const at::cuda::CUDAGuard guard(A.device());
  TORCH_CHECK(A.dim() == 3 && B.dim() == 3 && D.dim() == 3, "gemm_batched expects 3-D tensors");
  TORCH_CHECK(A.size(0) == B.size(0) && A.size(0) == D.size(0), "batch mismatch");
  for (const auto* t : {&A, &B}) {
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == torch::kBFloat16 && t->stride(2) == 1, "operands: bf16, row-major");
  }
  TORCH_CHECK(D.stride(2) == 1 && (D.scalar_type() == torch::kBFloat16 || D.scalar_type() == torch::kFloat32),
              "D must be bf16/fp32 row-major");
  GemmArgs a{};
  a.A = A.data_ptr();
  a.lda = A.stride(1);
  a.a_mn = a_kmajor ? 0 : 1;
  a.M = a_kmajor ? A.size(1) : A.size(2);
  a.K = a_kmajor ? A.size(2) : A.size(1);
  a.D = D.data_ptr();
  a.ldd = D.stride(1);
  a.d_fp32 = D.scalar_type() == torch::kFloat32;
  a.b_mn = b_kmajor ? 0 : 1;
  a.n_groups = 1;
  GemmGroup& gr = a.groups[0];
  gr.B = B.data_ptr();
  gr.ldb = B.stride(1);
  gr.n = b_kmajor ? B.size(1) : B.size(2);
  gr.k = b_kmajor ? B.size(2) : B.size(1);
  gr.row_begin = 0;
  gr.row_end = a.M;
  gr.bias = nullptr;
  TORCH_CHECK(gr.k == a.K, "K mismatch");
  TORCH_CHECK(D.size(1) >= a.M && D.size(2) >= gr.n, "D too small");
  a.batch = A.size(0);
  a.a_bstride = A.stride(0);
  a.b_bstride = B.stride(0);
  a.d_bstride = D.stride(0);
  a.alpha = (float)alpha;
  a.beta = (float)beta;
  if (C.has_value() && beta != 0.0) {
    const auto& c = C.value();
    TORCH_CHECK(c.dim() == 3 && c.stride(2) == 1 &&
                    (c.scalar_type() == torch::kBFloat16 || c.scalar_type() == torch::kFloat32),
                "C must be a row-major bf16/fp32 3-D tensor");
    a.C = c.data_ptr();
    a.ldc = c.stride(1);
    a.c_bstride = c.stride(0);
    a.c_fp32 = c.scalar_type() == torch::kFloat32;
  }
  check_launch(launch_gemm(a, stream()), "gemm_batched");
}

void gemm_grouped_nt(torch::Tensor A, std::vector<torch::Tensor> Bs, torch::Tensor D,
                     std::vector<c10::optional<torch::Tensor>> biases, c10::optional<torch::Tensor> gelu_pre,
                     std::vector<int64_t> bounds) {
  const at::cuda::CUDAGuard guard(A.device());
  TORCH_CHECK(bounds.size() == Bs.size() + 1, "bounds must have one more entry than weights");
  GemmArgs a = base_args(A, true, D);
  a.b_mn = 0;
  int G = 0;
  int prev_end = -1;
  for (size_t g = 0; g + 1 < bounds.size(); ++g) {
    if (bounds[g + 1] <= bounds[g]) continue;
    TORCH_CHECK(G < kGemmMaxGroups, "at most 4 groups");
    TORCH_CHECK(prev_end < 0 || prev_end == bounds[g], "row groups must be contiguous");
    TORCH_CHECK(bounds[g + 1] <= a.M, "row bounds beyond A");
    set_group(a, G, Bs[g], true, bounds[g], bounds[g + 1], g < biases.size() ? biases[g] : c10::nullopt);
    TORCH_CHECK(D.size(1) >= a.groups[G].n, "D too narrow");
    prev_end = bounds[g + 1];
    ++G;
  }
  if (G == 0) return;
  a.n_groups = G;
  if (gelu_pre.has_value()) {
    const auto& p = gelu_pre.value();
    TORCH_CHECK(p.scalar_type() == torch::kBFloat16 && p.stride(1) == 1, "gelu_pre must be bf16 row-major");
    a.epi = 1;
    a.aux = p.data_ptr();
    a.ldaux = p.stride(0);
  }
  check_launch(launch_gemm(a, stream()), "gemm_grouped_nt");
}

void gemm_dgelu(torch::Tensor dY, torch::Tensor Wd, torch::Tensor pre, torch::Tensor dpre, torch::Tensor post) {
  const at::cuda::CUDAGuard guard(dY.device());
  GemmArgs a = base_args(dY, true, dpre);
  a.b_mn = 1;
  a.n_groups = 1;
  set_group(a, 0, Wd, false, 0, a.M, c10::nullopt);
  TORCH_CHECK(a.groups[0].k == a.K, "K mismatch");
  TORCH_CHECK(pre.scalar_type() == torch::kBFloat16 && pre.stride(1) == 1 && post.stride(1) == 1, "bad pre/post");
  a.epi = 2;
  a.aux = pre.data_ptr();
  a.ldaux = pre.stride(0);
  a.aux2 = post.data_ptr();
  a.ldaux2 = post.stride(0);
  check_launch(launch_gemm(a, stream()), "gemm_dgelu");
}

// ------------------------------------------------------------------ QKV post-processing
std::vector<torch::Tensor> qkv_post_fwd(torch::Tensor raw, torch::Tensor qw, torch::Tensor kw, torch::Tensor cos_t,
                                        torch::Tensor sin_t, torch::Tensor itc, int64_t nv, int64_t na, int64_t heads,
                                        double eps) {
  const at::cuda::CUDAGuard guard(raw.device());
  check_bf16(raw, "raw");
  check_i32(itc, "interleave_to_concat");
  const int L = raw.size(0);
  const int HD = raw.size(1) / 3;
  const int D = HD / heads;
  TORCH_CHECK(cos_t.scalar_type() == torch::kFloat32 && cos_t.is_contiguous() && cos_t.size(0) >= L &&
                  cos_t.size(1) == D,
              "cos must be fp32 [L, D]");
  auto q = torch::empty({L, heads, D}, raw.options());
  auto k = torch::empty({L, heads, D}, raw.options());
  auto v = torch::empty({L, heads, D}, raw.options());
  check_launch(launch_qkv_post_fwd(raw.data_ptr(), qw.data_ptr<float>(), kw.data_ptr<float>(), cos_t.data_ptr<float>(),
                                   sin_t.data_ptr<float>(), itc.data_ptr<int>(), nv, na, L, heads, D, (float)eps,
                                   q.data_ptr(), k.data_ptr(), v.data_ptr(), stream()),
               "qkv_post_fwd");
  return {q, k, v};
}

std::vector<torch::Tensor> qkv_post_bwd(torch::Tensor dq, torch::Tensor dk, torch::Tensor dv, torch::Tensor raw,
                                        torch::Tensor qw, torch::Tensor kw, torch::Tensor cos_t, torch::Tensor sin_t,
                                        torch::Tensor itc, int64_t nv, int64_t na, int64_t heads, double eps) {
  const at::cuda::CUDAGuard guard(raw.device());
  check_bf16(dq, "dq");
  check_bf16(dk, "dk");
  check_bf16(dv, "dv");
  const int L = raw.size(0);
  const int HD = raw.size(1) / 3;
  const int D = HD / heads;
  auto draw = torch::empty_like(raw);
  auto dqw = torch::zeros({2 * D}, raw.options().dtype(torch::kFloat32));
  auto dkw = torch::zeros({2 * D}, raw.options().dtype(torch::kFloat32));
  check_launch(launch_qkv_post_bwd(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), raw.data_ptr(), qw.data_ptr<float>(),
                                   kw.data_ptr<float>(), cos_t.data_ptr<float>(), sin_t.data_ptr<float>(),
                                   itc.data_ptr<int>(), nv, na, L, heads, D, (float)eps, draw.data_ptr(),
                                   dqw.data_ptr<float>(), dkw.data_ptr<float>(), stream()),
               "qkv_post_bwd");
  return {draw, dqw, dkw};
}

// ------------------------------------------------------------------ attention
namespace {
void check_qkv(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == torch::kBFloat16 && t.dim() == 3 && t.is_contiguous(), name,
              " must be a contiguous bf16 CUDA [L, H, D] tensor");
}
}  // namespace

// items: int32 [n, 4] = (segment start, segment length, first row of the tile, 0)
std::vector<torch::Tensor> attn_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor items,
                                    int64_t n_valid, double scale) {
  const at::cuda::CUDAGuard guard(q.device());
  check_qkv(q, "q");
  check_qkv(k, "k");
  check_qkv(v, "v");
  check_i32(items, "items");
  const int L = q.size(0), H = q.size(1), D = q.size(2);
  auto o = torch::empty_like(q);
  auto lse = torch::empty({H, L}, q.options().dtype(torch::kFloat32));
  if (n_valid < L) o.narrow(0, n_valid, L - n_valid).zero_();
  check_launch(launch_attn_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), items.data_ptr<int>(), items.size(0), L, H, D,
                               (float)scale, o.data_ptr(), lse.data_ptr<float>(), stream()),
               "attn_fwd");
  return {o, lse};
}

std::vector<torch::Tensor> attn_bwd(torch::Tensor dout, torch::Tensor q, torch::Tensor k, torch::Tensor v,
                                    torch::Tensor o, torch::Tensor lse, torch::Tensor items_q, torch::Tensor items_kv,
                                    int64_t n_valid, double scale) {
  const at::cuda::CUDAGuard guard(q.device());
  check_qkv(dout, "dout");
  check_qkv(q, "q");
  check_qkv(o, "o");
  const int L = q.size(0), H = q.size(1), D = q.size(2);
  auto dq = torch::empty_like(q);
  auto dk = torch::empty_like(k);
  auto dv = torch::empty_like(v);
  if (n_valid < L) {
    dq.narrow(0, n_valid, L - n_valid).zero_();
    dk.narrow(0, n_valid, L - n_valid).zero_();
    dv.narrow(0, n_valid, L - n_valid).zero_();
  }
  auto delta = torch::empty({H, L}, q.options().dtype(torch::kFloat32));
  auto dq_acc = torch::empty({L, H, D}, q.options().dtype(torch::kFloat32));
  check_launch(launch_attn_bwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), dout.data_ptr(),
                               lse.data_ptr<float>(), items_q.data_ptr<int>(), items_q.size(0),
                               items_kv.data_ptr<int>(), items_kv.size(0), L, H, D, (float)scale,
                               delta.data_ptr<float>(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(),
                               dq_acc.data_ptr<float>(), stream()),
               "attn_bwd");
  return {dq, dk, dv};
}

// ------------------------------------------------------------------ Ulysses all-to-all fused in
namespace {
const uint64_t* peer_table(const torch::Tensor& t, int64_t cp, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == torch::kInt64 && t.is_contiguous() && t.numel() == cp, name,
              " must be a CUDA int64 [cp] table of peer addresses");
  return reinterpret_cast<const uint64_t*>(t.data_ptr<int64_t>());
}
}  // namespace

// qkv_post forward whose q/k/v rows go straight to their head owners' buffers (tables: [cp] int64).
void qkv_post_fwd_scatter(torch::Tensor raw, torch::Tensor qw, torch::Tensor kw, torch::Tensor cos_t,
                          torch::Tensor sin_t, torch::Tensor itc, int64_t nv, int64_t na, int64_t heads, double eps,
                          torch::Tensor peer_q, torch::Tensor peer_k, torch::Tensor peer_v, int64_t cp, int64_t rank) {
  const at::cuda::CUDAGuard guard(raw.device());
  check_rows(raw, "raw");
  check_i32(itc, "itc");
  const int L = raw.size(0);
  const int HD = raw.size(1) / 3;
  const int D = HD / heads;
  TORCH_CHECK(cos_t.scalar_type() == torch::kFloat32 && cos_t.is_contiguous() && cos_t.size(0) >= L &&
                  cos_t.size(1) == D,
              "cos must be fp32 [L, D]");
  check_launch(launch_qkv_post_fwd(raw.data_ptr(), qw.data_ptr<float>(), kw.data_ptr<float>(), cos_t.data_ptr<float>(),
                                   sin_t.data_ptr<float>(), itc.data_ptr<int>(), nv, na, L, heads, D, (float)eps,
                                   nullptr, nullptr, nullptr, stream(), peer_table(peer_q, cp, "peer_q"),
                                   peer_table(peer_k, cp, "peer_k"), peer_table(peer_v, cp, "peer_v"), (int)cp,
                                   (int)rank),
               "qkv_post_fwd_scatter");
}

// attention forward over the full sequence for this rank's heads; O is also written to its token
// owners (o_peer: [cp] int64 addresses of each rank's [rows, H_total, D] buffer).
std::vector<torch::Tensor> attn_fwd_cp(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor items,
                                       int64_t n_valid, double scale, torch::Tensor o_peer, int64_t cp,
                                       int64_t head_base, int64_t H_total) {
  const at::cuda::CUDAGuard guard(q.device());
  check_qkv(q, "q");
  check_qkv(k, "k");
  check_qkv(v, "v");
  check_i32(items, "items");
  const int L = q.size(0), H = q.size(1), D = q.size(2);
  auto o = torch::empty_like(q);
  auto lse = torch::empty({H, L}, q.options().dtype(torch::kFloat32));
  if (n_valid < L) o.narrow(0, n_valid, L - n_valid).zero_();
  check_launch(launch_attn_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), items.data_ptr<int>(), items.size(0), L, H, D,
                               (float)scale, o.data_ptr(), lse.data_ptr<float>(), stream(),
                               peer_table(o_peer, cp, "o_peer"), (int)cp, (int)head_base, (int)H_total),
               "attn_fwd_cp");
  return {o, lse};
}

// attention backward over the full sequence for this rank's heads: dO is read from the token
// owners, dQ / dK / dV are written to them.  Returns the gathered head-sharded dO.
torch::Tensor attn_bwd_cp(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor o, torch::Tensor lse,
                          torch::Tensor items_kv, int64_t n_valid, double scale, torch::Tensor do_peer,
                          torch::Tensor dq_peer, torch::Tensor dk_peer, torch::Tensor dv_peer, int64_t cp,
                          int64_t head_base, int64_t H_total) {
  const at::cuda::CUDAGuard guard(q.device());
  check_qkv(q, "q");
  check_qkv(k, "k");
  check_qkv(v, "v");
  check_qkv(o, "o");
  check_i32(items_kv, "items_kv");
  const int L = q.size(0), H = q.size(1), D = q.size(2);
  auto dout = torch::empty_like(q);
  auto delta = torch::empty({H, L}, q.options().dtype(torch::kFloat32));
  auto dq_acc = torch::empty({L, H, D}, q.options().dtype(torch::kFloat32));
  check_launch(launch_attn_bwd_cp(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr<float>(),
                                  items_kv.data_ptr<int>(), items_kv.size(0), L, H, D, (float)scale, (int)n_valid,
                                  delta.data_ptr<float>(), dout.data_ptr(), dq_acc.data_ptr<float>(),
                                  peer_table(do_peer, cp, "do_peer"), peer_table(dq_peer, cp, "dq_peer"),
                                  peer_table(dk_peer, cp, "dk_peer"), peer_table(dv_peer, cp, "dv_peer"), (int)cp,
                                  (int)head_base, (int)H_total, stream()),
               "attn_bwd_cp");
  return dout;
}

// ------------------------------------------------------------------ optimizer
namespace {
void check_half16(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.element_size() == 2 && t.is_contiguous(), name, " must be a contiguous 16-bit CUDA tensor");
}
const float* opt_ptr(const c10::optional<torch::Tensor>& t) { return t.has_value() ? t.value().data_ptr<float>() : nullptr; }
}  // namespace

// partial sums of squares of x (bf16 or fp32) appended into `partial` (fp32 [n_part]).
void sumsq_partial(torch::Tensor x, torch::Tensor partial) {
  const at::cuda::CUDAGuard guard(x.device());
  TORCH_CHECK(x.is_contiguous() && (x.scalar_type() == torch::kBFloat16 || x.scalar_type() == torch::kFloat32), "x");
  TORCH_CHECK(partial.scalar_type() == torch::kFloat32 && partial.is_contiguous(), "partial must be fp32");
  if (x.numel() == 0) {
    partial.zero_();
    return;
  }
  launch_sumsq(x.data_ptr(), x.scalar_type() == torch::kFloat32, x.numel(), partial.data_ptr<float>(),
               partial.numel(), stream());
  check_launch(nullptr, "sumsq");
}

// out[0] = sqrt(sum(partials)), out[1] = min(1, max_norm / (out[0] + 1e-6))
void norm_and_clip(torch::Tensor partials, double max_norm, torch::Tensor out) {
  const at::cuda::CUDAGuard guard(partials.device());
  launch_reduce_clip(partials.data_ptr<float>(), partials.numel(), (float)max_norm, out.data_ptr<float>(), stream());
  check_launch(nullptr, "norm_and_clip");
}

void muon_momentum(torch::Tensor buf, torch::Tensor g, c10::optional<torch::Tensor> clip, double mu, torch::Tensor u) {
  const at::cuda::CUDAGuard guard(buf.device());
  TORCH_CHECK(buf.scalar_type() == torch::kFloat32 && buf.is_contiguous() && g.is_contiguous() && u.is_contiguous(),
              "muon_momentum: contiguous fp32 buffer");
  TORCH_CHECK(buf.numel() == g.numel() && u.numel() == g.numel(), "muon_momentum: size mismatch");
  launch_muon_momentum(buf.data_ptr<float>(), g.data_ptr(), g.scalar_type() == torch::kFloat32, opt_ptr(clip),
                       (float)mu, g.numel(), u.data_ptr(), stream());
  check_launch(nullptr, "muon_momentum");
}

void muon_update(torch::Tensor hi, torch::Tensor lo, torch::Tensor u, torch::Tensor lr, double lr_scale, double wd) {
  const at::cuda::CUDAGuard guard(hi.device());
  check_half16(hi, "hi");
  check_half16(lo, "lo");
  TORCH_CHECK(u.numel() == hi.numel() && lo.numel() == hi.numel(), "muon_update: size mismatch");
  launch_muon_update(hi.data_ptr(), lo.data_ptr(), u.data_ptr(), lr.data_ptr<float>(), (float)lr_scale, (float)wd,
                     hi.numel(), stream());
  check_launch(nullptr, "muon_update");
}

// Muon update whose orthogonalised rows are read from `u_addr`: an address in this or another
// rank's peer-mapped memory (distributed Muon's scatter fused into the update).
void muon_update_peer(torch::Tensor hi, torch::Tensor lo, int64_t u_addr, torch::Tensor lr, double lr_scale,
                      double wd) {
  const at::cuda::CUDAGuard guard(hi.device());
  check_half16(hi, "hi");
  check_half16(lo, "lo");
  TORCH_CHECK(lo.numel() == hi.numel(), "muon_update_peer: size mismatch");
  TORCH_CHECK(u_addr != 0 && u_addr % 16 == 0, "muon_update_peer: u address must be 16-byte aligned");
  launch_muon_update(hi.data_ptr(), lo.data_ptr(), reinterpret_cast<const void*>(u_addr), lr.data_ptr<float>(),
                     (float)lr_scale, (float)wd, hi.numel(), stream());
  check_launch(nullptr, "muon_update_peer");
}

void adamw_update(torch::Tensor hi, torch::Tensor lo, torch::Tensor g, torch::Tensor m, torch::Tensor v,
                  c10::optional<torch::Tensor> clip, torch::Tensor lr, double beta1, double beta2, double eps,
                  double wd, int64_t step) {
  const at::cuda::CUDAGuard guard(hi.device());
  check_half16(hi, "hi");
  check_half16(lo, "lo");
  TORCH_CHECK(g.numel() == hi.numel() && m.numel() == hi.numel() && v.numel() == hi.numel(), "adamw: size mismatch");
  const double bc1 = 1.0 - std::pow(beta1, (double)step);
  const double bc2 = 1.0 - std::pow(beta2, (double)step);
  launch_adamw_update(hi.data_ptr(), lo.data_ptr(), g.data_ptr(), g.scalar_type() == torch::kFloat32,
                      m.data_ptr<float>(), v.data_ptr<float>(), opt_ptr(clip), lr.data_ptr<float>(), (float)beta1,
                      (float)beta2, (float)eps, (float)wd, (float)bc1, (float)std::sqrt(bc2), hi.numel(), stream());
  check_launch(nullptr, "adamw_update");
}

void split_master(torch::Tensor x, torch::Tensor hi, torch::Tensor lo) {
  const at::cuda::CUDAGuard guard(x.device());
  TORCH_CHECK(x.scalar_type() == torch::kFloat32 && x.is_contiguous() && x.numel() == hi.numel(), "split_master");
  launch_split_master(x.data_ptr<float>(), hi.data_ptr(), lo.data_ptr(), x.numel(), stream());
  check_launch(nullptr, "split_master");
}

void join_master(torch::Tensor hi, torch::Tensor lo, torch::Tensor x) {
  const at::cuda::CUDAGuard guard(x.device());
  TORCH_CHECK(x.scalar_type() == torch::kFloat32 && x.is_contiguous() && x.numel() == hi.numel(), "join_master");
  launch_join_master(hi.data_ptr(), lo.data_ptr(), x.data_ptr<float>(), x.numel(), stream());
  check_launch(nullptr, "join_master");
}

// Newton-Schulz helpers over a batch of M x M Gram matrices
void ns_trace(torch::Tensor R, torch::Tensor out) {
  const at::cuda::CUDAGuard guard(R.device());
  TORCH_CHECK(R.scalar_type() == torch::kFloat32 && R.dim() == 3 && R.is_contiguous(), "R must be fp32 [B, M, M]");
  launch_trace(R.data_ptr<float>(), R.size(0), R.size(1), out.data_ptr<float>(), stream());
  check_launch(nullptr, "ns_trace");
}
// The two per-element passes below move 16-byte vectors: contiguous [B, M, M] with M * M % 8 == 0
static void check_gram_batch(const torch::Tensor& t, torch::ScalarType dt, const char* what) {
  TORCH_CHECK(t.scalar_type() == dt && t.dim() == 3 && t.is_contiguous() && t.size(1) == t.size(2), what,
              " must be a contiguous [B, M, M] tensor of the expected dtype");
  TORCH_CHECK((t.size(1) * t.size(2)) % 8 == 0, what, ": M * M must be a multiple of 8");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0, what, " must be 16-byte aligned");
}
void ns_gram_normalize(torch::Tensor R, torch::Tensor norm2, double eps, torch::Tensor Rn) {
  const at::cuda::CUDAGuard guard(R.device());
  check_gram_batch(R, torch::kFloat32, "R");
  check_gram_batch(Rn, torch::kBFloat16, "Rn");
  TORCH_CHECK(Rn.sizes() == R.sizes() && norm2.numel() == R.size(0), "Rn / norm2 do not match R");
  launch_gram_normalize(R.data_ptr<float>(), norm2.data_ptr<float>(), R.size(0), R.size(1), (float)eps, Rn.data_ptr(),
                        stream());
  check_launch(nullptr, "ns_gram_normalize");
}
void ns_add_diag(torch::Tensor Z, double a) {
  const at::cuda::CUDAGuard guard(Z.device());
  launch_add_diag(Z.data_ptr(), Z.size(0), Z.size(1), (float)a, stream());
  check_launch(nullptr, "ns_add_diag");
}
void ns_scale_by_invnorm(torch::Tensor Q, torch::Tensor norm2, double eps) {
  const at::cuda::CUDAGuard guard(Q.device());
  check_gram_batch(Q, torch::kBFloat16, "Q");
  TORCH_CHECK(norm2.numel() == Q.size(0), "norm2 does not match Q");
  launch_scale_by_invnorm(Q.data_ptr(), norm2.data_ptr<float>(), Q.size(0), Q.size(1), (float)eps, stream());
  check_launch(nullptr, "ns_scale_by_invnorm");
}

int error_flag(bool reset) {
  return gemm_error_flag(reset) | packed_ops_error_flag(reset) | attn_error_flag(reset) | comm_error_flag(reset) |
         qkv_bounds_error(reset);
}

// ---------------------------------------------------------------- peer-memory collectives
void symm_barrier(torch::Tensor pads, int64_t rank, int64_t world, int64_t epoch, int64_t channel,
                  int64_t timeout_ms) {
  TORCH_CHECK(pads.is_cuda() && pads.scalar_type() == torch::kInt64 && pads.numel() >= world, "pads: int64 [world]");
  check_launch(launch_symm_barrier(reinterpret_cast<const uint64_t*>(pads.data_ptr<int64_t>()), (int)rank, (int)world,
                                   (uint32_t)epoch, (int)channel, (int)timeout_ms, stream()),
               "symm_barrier");
}

// segs: int64 [n, 3] (src, dst, n elements); prefix: int64 [n] work-unit prefix; seg_peer: int32 [n]
void peer_gather(torch::Tensor peers, torch::Tensor segs, torch::Tensor seg_peer, torch::Tensor prefix, int64_t total,
                 torch::Tensor out) {
  TORCH_CHECK(out.scalar_type() == torch::kBFloat16 && out.is_contiguous(), "peer_gather: bf16 contiguous output");
  check_launch(launch_peer_gather(reinterpret_cast<const uint64_t*>(peers.data_ptr<int64_t>()), segs.data_ptr<int64_t>(),
                                  seg_peer.data_ptr<int32_t>(), reinterpret_cast<const long long*>(prefix.data_ptr<int64_t>()),
                                  (int)segs.size(0), total,
                                  out.data_ptr(), stream()),
               "peer_gather");
}

void peer_reduce(torch::Tensor peers, int64_t world, torch::Tensor segs, torch::Tensor prefix, int64_t total,
                 double scale, torch::Tensor out) {
  TORCH_CHECK(out.scalar_type() == torch::kFloat32 && out.is_contiguous(), "peer_reduce: fp32 contiguous output");
  check_launch(launch_peer_reduce(reinterpret_cast<const uint64_t*>(peers.data_ptr<int64_t>()), (int)world,
                                  segs.data_ptr<int64_t>(), reinterpret_cast<const long long*>(prefix.data_ptr<int64_t>()),
                                  (int)segs.size(0), total, (float)scale, out.data_ptr<float>(), stream()),
               "peer_reduce");
}

// y [k, N] = a [k, K] @ W^T + bias, W row-sharded over the peers (rows_per_rank rows each, at element
// offset w_off of every peer's buffer)
void peer_gemv(torch::Tensor peers, int64_t w_off, int64_t rows_per_rank, torch::Tensor a,
               c10::optional<torch::Tensor> bias, torch::Tensor y) {
  const at::cuda::CUDAGuard guard(a.device());
  TORCH_CHECK(a.scalar_type() == torch::kBFloat16 && a.dim() == 2 && a.is_contiguous(), "peer_gemv: a must be bf16 [k, K]");
  TORCH_CHECK(y.scalar_type() == torch::kBFloat16 && y.dim() == 2 && y.is_contiguous() && y.size(0) == a.size(0),
              "peer_gemv: y must be bf16 [k, N]");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(a.data_ptr()) & 15) == 0, "peer_gemv: a must be 16-byte aligned");
  TORCH_CHECK(peers.scalar_type() == torch::kInt64 && peers.is_cuda(), "peer_gemv: peers must be a device int64 array");
  TORCH_CHECK(rows_per_rank > 0 && (y.size(1) + rows_per_rank - 1) / rows_per_rank <= peers.numel(),
              "peer_gemv: the rows do not fit the ranks");
  const void* b = nullptr;
  if (bias.has_value() && bias->defined()) {
    TORCH_CHECK(bias->scalar_type() == torch::kBFloat16 && bias->numel() == y.size(1) && bias->is_contiguous(),
                "peer_gemv: bias must be bf16 [N]");
    b = bias->data_ptr();
  }
  int dev = a.device().index(), sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  check_launch(launch_peer_gemv(reinterpret_cast<const uint64_t*>(peers.data_ptr<int64_t>()), w_off, (int)rows_per_rank,
                                (int)y.size(1), (int)a.size(1), (int)a.size(0), a.data_ptr(), b, y.data_ptr(), sms,
                                stream()),
               "peer_gemv");
}

}  // namespace pan

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "pan2_b200 sm_100a kernels";
  // Every binding releases the GIL while it runs (arguments are converted first): a launch that
  // blocks on a full stream queue, e.g. the deferred optimizer's enqueue thread, must not stall the
  // Python thread that enqueues the forward.  No binding touches Python objects.
  const auto kNoGil = py::call_guard<py::gil_scoped_release>();
  m.def("ln_modulate_fwd", &pan::ln_modulate_fwd, kNoGil);
  m.def("ln_modulate_bwd", &pan::ln_modulate_bwd, kNoGil);
  m.def("gate_residual_fwd", &pan::gate_residual_fwd, kNoGil);
  m.def("gate_bwd", &pan::gate_bwd, kNoGil);
  m.def("simple_concat_fwd", &pan::simple_concat_fwd, kNoGil);
  m.def("segment_sum", &pan::segment_sum, kNoGil);
  m.def("column_sum", &pan::column_sum, kNoGil);
  m.def("mse_fwd", &pan::mse_fwd, kNoGil);
  m.def("mse_bwd", &pan::mse_bwd, kNoGil);
  m.def("gather_rows", &pan::gather_rows, kNoGil);
  m.def("gemm", &pan::gemm, kNoGil);
  m.def("gemm_force_cta_group", &pan::gemm_force_cta_group, kNoGil);
  m.def("attn_set_forward_variant", &pan::attn_set_forward_variant, kNoGil);
  m.def("attn_get_variant", &pan::attn_get_variant, kNoGil);
  m.def("gemm_tuning", &pan::gemm_tuning, kNoGil);
  m.def("gemm_grouped_nt", &pan::gemm_grouped_nt, kNoGil);
  m.def("gemm_batched", &pan::gemm_batched, kNoGil);
  m.def("gemm_dgelu", &pan::gemm_dgelu, kNoGil);
  m.def("qkv_post_fwd", &pan::qkv_post_fwd, kNoGil);
  m.def("qkv_post_bwd", &pan::qkv_post_bwd, kNoGil);
  m.def("attn_fwd", &pan::attn_fwd, kNoGil);
  m.def("attn_bwd", &pan::attn_bwd, kNoGil);
  m.def("qkv_post_fwd_scatter", &pan::qkv_post_fwd_scatter, kNoGil);
  m.def("attn_fwd_cp", &pan::attn_fwd_cp, kNoGil);
  m.def("attn_bwd_cp", &pan::attn_bwd_cp, kNoGil);
  m.def("sumsq_partial", &pan::sumsq_partial, kNoGil);
  m.def("norm_and_clip", &pan::norm_and_clip, kNoGil);
  m.def("muon_momentum", &pan::muon_momentum, kNoGil);
  m.def("muon_update", &pan::muon_update, kNoGil);
  m.def("muon_update_peer", &pan::muon_update_peer, kNoGil);
  m.def("adamw_update", &pan::adamw_update, kNoGil);
  m.def("split_master", &pan::split_master, kNoGil);
  m.def("join_master", &pan::join_master, kNoGil);
  m.def("ns_trace", &pan::ns_trace, kNoGil);
  m.def("ns_gram_normalize", &pan::ns_gram_normalize, kNoGil);
  m.def("ns_add_diag", &pan::ns_add_diag, kNoGil);
  m.def("ns_scale_by_invnorm", &pan::ns_scale_by_invnorm, kNoGil);
  m.def("error_flag", &pan::error_flag, py::arg("reset") = true, kNoGil);
  m.def("symm_barrier", &pan::symm_barrier, kNoGil);
  m.def("peer_gather", &pan::peer_gather, kNoGil);
  m.def("peer_reduce", &pan::peer_reduce, kNoGil);
  m.def("peer_gemv", &pan::peer_gemv, kNoGil);
}
