// Plain-C++ launch interface of the sm_100a kernels.  The .cu files implement these with raw
// pointers and a CUDA stream; bindings.cpp (the only file that includes torch headers) validates
// tensors, allocates outputs and calls them.  Keeping torch out of nvcc's translation units keeps
// kernel rebuilds to seconds.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace pan {

// ------------------------------------------------------------------ packed_ops.cu
void launch_ln_modulate_fwd(const void* x, const float* stats, const void* shift, const void* scale,
                            const int* bounds, int n_seg, int L, int C, void* y, cudaStream_t s);
void launch_ln_modulate_bwd(const void* g, const void* x, const float* stats, const void* scale, const int* bounds,
                            int n_seg, int L, int C, void* dx, float* dshift, float* dscale, cudaStream_t s);
void launch_gate_residual_fwd(const void* y, const void* gate, const void* res, const int* bounds, int n_seg, int L,
                              int C, void* out, float* stats, cudaStream_t s);
void launch_gate_bwd(const void* g, const void* y, const void* gate, const int* bounds, int n_seg, int L, int C,
                     void* dy, float* dgate, cudaStream_t s);
void launch_concat_fwd(const void* vid, const void* txt, const void* ttv, int nv, int nt, int L, int C, void* out,
                       float* stats, cudaStream_t s);
void launch_segment_sum(const void* x, const int* bounds, int n_seg, int L, int C, float* out, cudaStream_t s);
void launch_mse_fwd(const void* pred, const void* tgt, size_t n, float* partial, int n_part, float* out,
                    cudaStream_t s);
void launch_mse_bwd(const void* pred, const void* tgt, const float* gsum, size_t n, size_t total, void* dpred,
                    cudaStream_t s);
void launch_gather_rows(const void* x, const int* idx, int rows, int vec16_per_row, void* out, cudaStream_t s);
int packed_ops_error_flag(bool reset);

// ------------------------------------------------------------------ gemm_sm100.cu
constexpr int kGemmMaxGroups = 4;
struct GemmGroup {
  const void* B;         // bf16, row-major; K-major [N, K] or MN-major [K, N]
  long long ldb;         // row stride of B (elements)
  int n;                 // N of this group
  int k;                 // K of this group (<= A's K)
  int row_begin, row_end;  // rows of A / D handled by this group
  const void* bias;      // bf16 [N] or null
};
struct GemmArgs {
  const void* A;         // bf16 row-major; K-major [M, K] or MN-major [K, M]
  long long lda;
  int M, K;              // logical A extents
  int a_mn, b_mn;
  int n_groups;
  GemmGroup groups[kGemmMaxGroups];
  void* D;               // bf16 or fp32 row-major [M, >= N]
  long long ldd;
  int d_fp32;
  int epi;               // 0 plain, 1 GELU (aux <- pre-activation), 2 dGELU (aux = pre in, aux2 <- GELU(pre))
  void* aux;
  long long ldaux;
  void* aux2;
  long long ldaux2;
  int accumulate;        // D += ...  (same as C = D, beta = 1)
  // batched: `batch` problems with element strides between consecutive A / B / D / C matrices
  int batch = 1;
  long long a_bstride = 0, b_bstride = 0, d_bstride = 0;
  // out = alpha * acc + beta * C (+ bias)
  float alpha = 1.f, beta = 0.f;
  const void* C = nullptr;
  long long ldc = 0, c_bstride = 0;
  int c_fp32 = 0;
};
// Returns an error string (nullptr on success).
const char* launch_gemm(const GemmArgs& args, cudaStream_t s);
int gemm_error_flag(bool reset);
// 0: CTA pairs or single CTAs chosen per launch; 1 / 2: forced.
void gemm_force_cta_group(int cg);
// CTA-pair smem stages (4 or 6), timing-probe bits (0 in normal use) and the M-band budget in MB
// of the tile order (0: N bands only).
void gemm_tuning(int pair_stages, int probe, int band_mb, int band_n);

// ------------------------------------------------------------------ comm_ops.cu (peer memory)
const char* launch_symm_barrier(const uint64_t* pads, int rank, int world, uint32_t epoch, int channel,
                                int timeout_ms, cudaStream_t s);
const char* launch_peer_gather(const uint64_t* peers, const void* segs, const int* seg_peer, const long long* prefix,
                               int n_seg, long long total, void* out, cudaStream_t s);
const char* launch_peer_reduce(const uint64_t* peers, int world, const void* segs, const long long* prefix, int n_seg,
                               long long total, float scale, float* out, cudaStream_t s);
const char* launch_peer_gemv(const uint64_t* peers, long long w_off, int rows_per_rank, int N, int K, int k,
                             const void* a, const void* bias, void* y, int n_sms, cudaStream_t s);
int comm_error_flag(bool reset);

}  // namespace pan
