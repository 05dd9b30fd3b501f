// Optimizer kernels (sm_100a) over flat parameter shards.
//
// Master weights are exact fp32 values stored as two 16-bit halves: `hi` (the upper 16 bits, a bf16
// that the GEMMs read directly as the compute weight) and `lo` (the lower 16 bits).  Joining them
// gives back the fp32 bit pattern exactly, so the optimizer updates fp32 masters with no extra
// bf16 copy of the weights.  The learning rate and the gradient-clip coefficient are device
// scalars, so a step never waits on the host.
//
//   muon_momentum : buf = mu*buf + (1-mu)*g*clip ;  u = (1-mu)*g*clip + mu*buf  (Nesterov, bf16 u)
//                   -- the reference's _muon_momentum_nesterov_kernel (pan/optim/muon_triton.py:25-51)
//   muon_update   : p = p*(1 - lr*wd) - lr*adj*u          (muon_triton.py:111-161)
//   adamw_update  : torch.optim.AdamW semantics (decoupled decay, bias corrections), fp32 m/v
//   sumsq         : per-CTA partial sums of g^2 for the global gradient norm
//   clip_coef     : clip = min(1, max_norm / (sqrt(sum) + 1e-6)) on the device
#include "common.cuh"
#include "launchers.h"

namespace pan {
namespace {

__device__ __forceinline__ float join_master(uint16_t hi, uint16_t lo) {
  return __uint_as_float(((uint32_t)hi << 16) | lo);
}
__device__ __forceinline__ void split_master(float x, uint16_t& hi, uint16_t& lo) {
  const uint32_t b = __float_as_uint(x);
  hi = (uint16_t)(b >> 16);
  lo = (uint16_t)(b & 0xFFFFu);
}

template <typename G>
__device__ __forceinline__ float to_f(G g);
template <>
__device__ __forceinline__ float to_f<float>(float g) { return g; }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 g) { return __bfloat162float(g); }

template <typename G>
__global__ void sumsq_kernel(const G* __restrict__ x, size_t n, float* __restrict__ partial) {
  float acc = 0.f;
  constexpr int V = 16 / sizeof(G);  // elements per 16-byte load
  const size_t nv = (reinterpret_cast<uintptr_t>(x) % 16 == 0) ? n / V : 0;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < nv; i += stride) {
    const uint4 raw = reinterpret_cast<const uint4*>(x)[i];
    const G* e = reinterpret_cast<const G*>(&raw);
#pragma unroll
    for (int k = 0; k < V; ++k) {
      const float v = to_f<G>(e[k]);
      acc += v * v;
    }
  }
  for (size_t i = nv * V + (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const float v = to_f<G>(x[i]);
    acc += v * v;
  }
  acc = warp_sum(acc);
  __shared__ float ws[32];
  if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? ws[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) partial[blockIdx.x] = v;
  }
}

// sum of `n` partials into out[0] (deterministic single CTA), then clip coefficient into out[1]
__global__ void reduce_clip_kernel(const float* __restrict__ partial, int n, float max_norm, float* __restrict__ out) {
  float acc = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) acc += partial[i];
  acc = warp_sum(acc);
  __shared__ float ws[32];
  if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? ws[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) {
      const float norm = sqrtf(v);
      out[0] = norm;
      out[1] = max_norm > 0.f ? fminf(1.f, max_norm / (norm + 1e-6f)) : 1.f;
    }
  }
}

template <typename G>
__global__ void muon_momentum_kernel(float* __restrict__ buf, const G* __restrict__ g, const float* __restrict__ clip,
                                     float mu, size_t n, __nv_bfloat16* __restrict__ u) {
  const float c = clip ? clip[0] : 1.f;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const float gi = to_f<G>(g[i]) * c;
    const float b = mu * buf[i] + (1.f - mu) * gi;
    buf[i] = b;
    u[i] = __float2bfloat16_rn((1.f - mu) * gi + mu * b);
  }
}

__global__ void muon_update_kernel(uint16_t* __restrict__ hi, uint16_t* __restrict__ lo,
                                   const __nv_bfloat16* __restrict__ u, const float* __restrict__ lr, float lr_scale,
                                   float wd, size_t n) {
  const float l = lr[0];
  const float decay = 1.f - l * wd;
  const float step = l * lr_scale;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    float p = join_master(hi[i], lo[i]);
    p = p * decay - step * __bfloat162float(u[i]);
    split_master(p, hi[i], lo[i]);
  }
}

// Same update, 8 elements per thread with 16-byte loads of u (which may be another rank's memory,
// read over NVLink: the scatter of distributed Muon's orthogonalised rows fused into the update).
__global__ void muon_update_vec_kernel(uint16_t* __restrict__ hi, uint16_t* __restrict__ lo,
                                       const __nv_bfloat16* __restrict__ u, const float* __restrict__ lr,
                                       float lr_scale, float wd, size_t n8) {
  const float l = lr[0];
  const float decay = 1.f - l * wd;
  const float step = l * lr_scale;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (size_t)gridDim.x * blockDim.x) {
    const uint4 uv = reinterpret_cast<const uint4*>(u)[i];
    uint4 hv = reinterpret_cast<const uint4*>(hi)[i];
    uint4 lv = reinterpret_cast<const uint4*>(lo)[i];
    const __nv_bfloat16* ub = reinterpret_cast<const __nv_bfloat16*>(&uv);
    uint16_t* hb = reinterpret_cast<uint16_t*>(&hv);
    uint16_t* lb = reinterpret_cast<uint16_t*>(&lv);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float p = join_master(hb[e], lb[e]);
      p = p * decay - step * __bfloat162float(ub[e]);
      split_master(p, hb[e], lb[e]);
    }
    reinterpret_cast<uint4*>(hi)[i] = hv;
    reinterpret_cast<uint4*>(lo)[i] = lv;
  }
}

template <typename G>
__global__ void adamw_update_kernel(uint16_t* __restrict__ hi, uint16_t* __restrict__ lo, const G* __restrict__ g,
                                    float* __restrict__ m, float* __restrict__ v, const float* __restrict__ clip,
                                    const float* __restrict__ lr, float beta1, float beta2, float eps, float wd,
                                    float bc1, float bc2_sqrt, size_t n) {
  const float c = clip ? clip[0] : 1.f;
  const float l = lr[0];
  const float decay = 1.f - l * wd;
  const float step = l / bc1;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const float gi = to_f<G>(g[i]) * c;
    const float mi = beta1 * m[i] + (1.f - beta1) * gi;
    const float vi = beta2 * v[i] + (1.f - beta2) * gi * gi;
    m[i] = mi;
    v[i] = vi;
    float p = join_master(hi[i], lo[i]) * decay;
    p -= step * mi / (sqrtf(vi) / bc2_sqrt + eps);
    split_master(p, hi[i], lo[i]);
  }
}

__global__ void split_kernel(const float* __restrict__ x, uint16_t* __restrict__ hi, uint16_t* __restrict__ lo,
                             size_t n) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    split_master(x[i], hi[i], lo[i]);
}

__global__ void join_kernel(const uint16_t* __restrict__ hi, const uint16_t* __restrict__ lo, float* __restrict__ x,
                            size_t n) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    x[i] = join_master(hi[i], lo[i]);
}

// R[b] diagonal sums: norm2[b] = trace(R[b]) for b < batch, R fp32 [batch, M, M]
__global__ void trace_kernel(const float* __restrict__ R, int M, long long bstride, float* __restrict__ out) {
  const int b = blockIdx.x;
  float acc = 0.f;
  for (int i = threadIdx.x; i < M; i += blockDim.x) acc += R[b * bstride + (size_t)i * M + i];
  acc = warp_sum(acc);
  __shared__ float ws[32];
  if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? ws[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) out[b] = v;
  }
}

// Rn[b] = bf16(R[b] / max(norm2[b], eps^2)).  `M * M` is a multiple of 8 (M of the Gram matrices
// is a multiple of 8), so each thread moves 32 bytes of fp32 in and one 16-byte bf16 vector out; the
// grid's y dimension walks the batch and x fills the SMs.
__global__ void gram_normalize_kernel(const float* __restrict__ R, const float* __restrict__ norm2, int M,
                                      float eps, __nv_bfloat16* __restrict__ Rn) {
  const int b = blockIdx.y;
  const float s = 1.f / fmaxf(norm2[b], eps * eps);
  const size_t off = (size_t)b * M * M;
  const size_t n8 = (size_t)M * M / 8;
  const float4* src = reinterpret_cast<const float4*>(R + off);
  uint4* dst = reinterpret_cast<uint4*>(Rn + off);
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (size_t)gridDim.x * blockDim.x) {
    const float4 a = src[2 * i], c = src[2 * i + 1];
    uint4 o;
    o.x = pack_bf16(a.x * s, a.y * s);
    o.y = pack_bf16(a.z * s, a.w * s);
    o.z = pack_bf16(c.x * s, c.y * s);
    o.w = pack_bf16(c.z * s, c.w * s);
    dst[i] = o;
  }
}

__global__ void add_diag_kernel(__nv_bfloat16* __restrict__ Z, int M, float a) {
  const int b = blockIdx.y;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < M; i += gridDim.x * blockDim.x) {
    __nv_bfloat16* p = Z + (size_t)b * M * M + (size_t)i * M + i;
    *p = __float2bfloat16_rn(__bfloat162float(*p) + a);
  }
}

// Q[b] *= 1 / sqrt(max(norm2[b], eps^2)), eight bf16 per 16-byte access (M * M % 8 == 0)
__global__ void scale_by_invnorm_kernel(__nv_bfloat16* __restrict__ Q, const float* __restrict__ norm2, int M,
                                        float eps) {
  const int b = blockIdx.y;
  const float s = rsqrtf(fmaxf(norm2[b], eps * eps));
  uint4* q = reinterpret_cast<uint4*>(Q + (size_t)b * M * M);
  const size_t n8 = (size_t)M * M / 8;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (size_t)gridDim.x * blockDim.x) {
    uint4 v = q[i];
    uint32_t* w = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[j]));
      w[j] = pack_bf16(f.x * s, f.y * s);
    }
    q[i] = v;
  }
}

// CTAs along x for a batched per-matrix pass of n8 16-byte vectors: about 16 CTAs per SM in total
inline dim3 batched_grid(int batch, size_t n8) {
  size_t per = (148 * 16 + batch - 1) / batch;
  size_t need = (n8 + 255) / 256;
  return dim3((unsigned)(need < per ? (need > 0 ? need : 1) : per), batch);
}

inline int grid_for(size_t n) {
  size_t b = (n + 255) / 256;
  return (int)(b < 148 * 16 ? (b > 0 ? b : 1) : 148 * 16);
}

}  // namespace

void launch_sumsq(const void* x, bool fp32, size_t n, float* partial, int n_part, cudaStream_t s) {
  if (fp32)
    sumsq_kernel<float><<<n_part, 256, 0, s>>>((const float*)x, n, partial);
  else
    sumsq_kernel<__nv_bfloat16><<<n_part, 256, 0, s>>>((const __nv_bfloat16*)x, n, partial);
}
void launch_reduce_clip(const float* partial, int n, float max_norm, float* out, cudaStream_t s) {
  reduce_clip_kernel<<<1, 1024, 0, s>>>(partial, n, max_norm, out);
}
void launch_muon_momentum(float* buf, const void* g, bool g_fp32, const float* clip, float mu, size_t n, void* u,
                          cudaStream_t s) {
  if (g_fp32)
    muon_momentum_kernel<float><<<grid_for(n), 256, 0, s>>>(buf, (const float*)g, clip, mu, n, (__nv_bfloat16*)u);
  else
    muon_momentum_kernel<__nv_bfloat16><<<grid_for(n), 256, 0, s>>>(buf, (const __nv_bfloat16*)g, clip, mu, n,
                                                                     (__nv_bfloat16*)u);
}
void launch_muon_update(void* hi, void* lo, const void* u, const float* lr, float lr_scale, float wd, size_t n,
                        cudaStream_t s) {
  const bool vec = n % 8 == 0 && ((reinterpret_cast<uintptr_t>(hi) | reinterpret_cast<uintptr_t>(lo) |
                                   reinterpret_cast<uintptr_t>(u)) & 15) == 0;
  if (vec)
    muon_update_vec_kernel<<<grid_for(n / 8), 256, 0, s>>>((uint16_t*)hi, (uint16_t*)lo, (const __nv_bfloat16*)u, lr,
                                                           lr_scale, wd, n / 8);
  else
    muon_update_kernel<<<grid_for(n), 256, 0, s>>>((uint16_t*)hi, (uint16_t*)lo, (const __nv_bfloat16*)u, lr,
                                                   lr_scale, wd, n);
}
void launch_adamw_update(void* hi, void* lo, const void* g, bool g_fp32, float* m, float* v, const float* clip,
                         const float* lr, float beta1, float beta2, float eps, float wd, float bc1, float bc2_sqrt,
                         size_t n, cudaStream_t s) {
  if (g_fp32)
    adamw_update_kernel<float><<<grid_for(n), 256, 0, s>>>((uint16_t*)hi, (uint16_t*)lo, (const float*)g, m, v, clip,
                                                           lr, beta1, beta2, eps, wd, bc1, bc2_sqrt, n);
  else
    adamw_update_kernel<__nv_bfloat16><<<grid_for(n), 256, 0, s>>>((uint16_t*)hi, (uint16_t*)lo,
                                                                   (const __nv_bfloat16*)g, m, v, clip, lr, beta1,
                                                                   beta2, eps, wd, bc1, bc2_sqrt, n);
}
void launch_split_master(const float* x, void* hi, void* lo, size_t n, cudaStream_t s) {
  split_kernel<<<grid_for(n), 256, 0, s>>>(x, (uint16_t*)hi, (uint16_t*)lo, n);
}
void launch_join_master(const void* hi, const void* lo, float* x, size_t n, cudaStream_t s) {
  join_kernel<<<grid_for(n), 256, 0, s>>>((const uint16_t*)hi, (const uint16_t*)lo, x, n);
}
void launch_trace(const float* R, int batch, int M, float* out, cudaStream_t s) {
  trace_kernel<<<batch, 256, 0, s>>>(R, M, (long long)M * M, out);
}
void launch_gram_normalize(const float* R, const float* norm2, int batch, int M, float eps, void* Rn, cudaStream_t s) {
  gram_normalize_kernel<<<batched_grid(batch, (size_t)M * M / 8), 256, 0, s>>>(R, norm2, M, eps, (__nv_bfloat16*)Rn);
}
void launch_add_diag(void* Z, int batch, int M, float a, cudaStream_t s) {
  dim3 grid((M + 255) / 256, batch);
  add_diag_kernel<<<grid, 256, 0, s>>>((__nv_bfloat16*)Z, M, a);
}
void launch_scale_by_invnorm(void* Q, const float* norm2, int batch, int M, float eps, cudaStream_t s) {
  scale_by_invnorm_kernel<<<batched_grid(batch, (size_t)M * M / 8), 256, 0, s>>>((__nv_bfloat16*)Q, norm2, M, eps);
}

}  // namespace pan
