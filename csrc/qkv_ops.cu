// QKV post-processing for the grouped QKV projection (sm_100a).
//
// Forward, per concat row p (video rows [0, nv), text rows [nv, na)) and head h:
//   Q/K: z = raw * w[mod] * rsqrt(mean(raw^2) + eps);  y = z * cos + rotate_half(z) * sin  (fp32)
//   V:   y = raw
// and row p is written to interleave row itc[p] of q/k/v [L, H, D] (bf16).  Interleave rows that
// no active concat row maps to (padding) are zeroed.  RoPE tables are indexed by interleave row.
// Same math as the reference's K13/K14 Triton kernels (pan/models/transformers/modules/
// triton_kernels.py:1201-1378) but in one pass with a single bf16 rounding.
//
// Backward, per concat row p: dz = rope^T(dy), dw += dz * raw * r, and
//   draw = r * w * dz - (r^3 / D) * raw * sum(dz * w * raw)      (RMS-norm Jacobian)
// (K15/K16, triton_kernels.py:1427-1624); V rows are gathered back.  One warp owns one row and
// walks its heads; each lane holds D/32 consecutive elements so RoPE pairs stay in-lane.
#include "common.cuh"
#include "launchers.h"

namespace pan {
namespace {

// Ulysses scatter of the forward outputs: when q/k/v are set they hold, per cp-rank, the address
// of that rank's head-sharded [S, hl, D] buffer (S = cp * local rows); local interleave row t of
// rank `rank` is global row t * cp + rank, and head h lives on rank h / hl as its head h % hl.
struct HeadScatter {
  const uint64_t* q;
  const uint64_t* k;
  const uint64_t* v;
  int cp, rank, hl;
};

template <int EPL>
__device__ __forceinline__ void loadv(const __nv_bfloat16* p, float (&v)[EPL]) {
  if (EPL == 4) {
    const uint2 r = *reinterpret_cast<const uint2*>(p);
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&r.x));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&r.y));
    v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
  } else {
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
    v[0] = a.x; v[1] = a.y;
  }
}

template <int EPL>
__device__ __forceinline__ void storev(__nv_bfloat16* p, const float (&v)[EPL]) {
  if (EPL == 4) {
    uint2 r;
    *reinterpret_cast<__nv_bfloat162*>(&r.x) = __floats2bfloat162_rn(v[0], v[1]);
    *reinterpret_cast<__nv_bfloat162*>(&r.y) = __floats2bfloat162_rn(v[2], v[3]);
    *reinterpret_cast<uint2*>(p) = r;
  } else {
    *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(v[0], v[1]);
  }
}

template <int EPL>
__global__ void qkv_post_fwd_kernel(const __nv_bfloat16* __restrict__ raw, const float* __restrict__ qw,
                                    const float* __restrict__ kw, const float* __restrict__ cos_t,
                                    const float* __restrict__ sin_t, const int* __restrict__ itc, int nv, int na,
                                    int L, int H, float eps, __nv_bfloat16* __restrict__ q, __nv_bfloat16* __restrict__ k,
                                    __nv_bfloat16* __restrict__ v, const HeadScatter hs) {
  constexpr int D = EPL * 32;
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  const int HD = H * D;
  for (int p = blockIdx.x * warps + (threadIdx.x >> 5); p < L; p += gridDim.x * warps) {
    const int dst = PAN_IDX(itc[p], L, 201);
    const size_t orow = (size_t)dst * HD;
    // destination of (this row, head h) in q / k / v: the local interleave row, or with the
    // Ulysses scatter on, row dst * cp + rank of head owner h / hl's head-sharded buffer
    auto out_at = [&](__nv_bfloat16* local, const uint64_t* tab, int h) -> __nv_bfloat16* {
      if (tab == nullptr) return local + orow + h * D + lane * EPL;
      const size_t g = (size_t)dst * hs.cp + hs.rank;
      return reinterpret_cast<__nv_bfloat16*>(tab[h / hs.hl]) + (g * hs.hl + h % hs.hl) * D + lane * EPL;
    };
    if (p >= na) {  // padding: zero the interleave row
      float z[EPL] = {};
      for (int h = 0; h < H; ++h) {
        storev<EPL>(out_at(q, hs.q, h), z);
        storev<EPL>(out_at(k, hs.k, h), z);
        storev<EPL>(out_at(v, hs.v, h), z);
      }
      continue;
    }
    const int mod = p < nv ? 0 : 1;
    float c[EPL], s[EPL], wq[EPL], wk[EPL];
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      c[i] = cos_t[(size_t)dst * D + lane * EPL + i];
      s[i] = sin_t[(size_t)dst * D + lane * EPL + i];
      wq[i] = qw[mod * D + lane * EPL + i];
      wk[i] = kw[mod * D + lane * EPL + i];
    }
    const __nv_bfloat16* rr = raw + (size_t)p * 3 * HD;
    for (int h = 0; h < H; ++h) {
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        float u[EPL];
        loadv<EPL>(rr + which * HD + h * D + lane * EPL, u);
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < EPL; ++i) ss += u[i] * u[i];
        const float r = rsqrtf(warp_sum(ss) / D + eps);
        float z[EPL], y[EPL];
#pragma unroll
        for (int i = 0; i < EPL; ++i) z[i] = u[i] * (which == 0 ? wq[i] : wk[i]) * r;
#pragma unroll
        for (int i = 0; i < EPL; i += 2) {
          y[i] = z[i] * c[i] - z[i + 1] * s[i];
          y[i + 1] = z[i + 1] * c[i + 1] + z[i] * s[i + 1];
        }
        storev<EPL>(which == 0 ? out_at(q, hs.q, h) : out_at(k, hs.k, h), y);
      }
      float vv[EPL];
      loadv<EPL>(rr + 2 * HD + h * D + lane * EPL, vv);
      storev<EPL>(out_at(v, hs.v, h), vv);
    }
  }
}

template <int EPL>
__global__ void qkv_post_bwd_kernel(const __nv_bfloat16* __restrict__ dq, const __nv_bfloat16* __restrict__ dk,
                                    const __nv_bfloat16* __restrict__ dv, const __nv_bfloat16* __restrict__ raw,
                                    const float* __restrict__ qw, const float* __restrict__ kw,
                                    const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                                    const int* __restrict__ itc, int nv, int na, int L, int H, float eps,
                                    __nv_bfloat16* __restrict__ draw, float* __restrict__ dqw,
                                    float* __restrict__ dkw) {
  constexpr int D = EPL * 32;
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  const int HD = H * D;
  // per-lane partial affine gradients: [modality][q/k][EPL]
  float acc[2][2][EPL] = {};
  for (int p = blockIdx.x * warps + (threadIdx.x >> 5); p < L; p += gridDim.x * warps) {
    __nv_bfloat16* dr = draw + (size_t)p * 3 * HD;
    if (p >= na) {
      float z[EPL] = {};
      for (int j = 0; j < 3 * H; ++j) storev<EPL>(dr + j * D + lane * EPL, z);
      continue;
    }
    const int src = PAN_IDX(itc[p], L, 202);
    const size_t irow = (size_t)src * HD;
    const int mod = p < nv ? 0 : 1;
    float c[EPL], s[EPL], wq[EPL], wk[EPL];
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      c[i] = cos_t[(size_t)src * D + lane * EPL + i];
      s[i] = sin_t[(size_t)src * D + lane * EPL + i];
      wq[i] = qw[mod * D + lane * EPL + i];
      wk[i] = kw[mod * D + lane * EPL + i];
    }
    const __nv_bfloat16* rr = raw + (size_t)p * 3 * HD;
    for (int h = 0; h < H; ++h) {
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        float u[EPL], dy[EPL], dz[EPL];
        loadv<EPL>(rr + which * HD + h * D + lane * EPL, u);
        loadv<EPL>((which == 0 ? dq : dk) + irow + h * D + lane * EPL, dy);
#pragma unroll
        for (int i = 0; i < EPL; i += 2) {
          dz[i] = dy[i] * c[i] + dy[i + 1] * s[i + 1];
          dz[i + 1] = dy[i + 1] * c[i + 1] - dy[i] * s[i];
        }
        float ss = 0.f, dot = 0.f;
#pragma unroll
        for (int i = 0; i < EPL; ++i) {
          const float w = which == 0 ? wq[i] : wk[i];
          ss += u[i] * u[i];
          dot += dz[i] * w * u[i];
        }
        ss = warp_sum(ss);
        dot = warp_sum(dot);
        const float r = rsqrtf(ss / D + eps);
        const float r3 = r * r * r / D;
        float du[EPL];
#pragma unroll
        for (int i = 0; i < EPL; ++i) {
          const float w = which == 0 ? wq[i] : wk[i];
          acc[mod][which][i] += dz[i] * u[i] * r;
          du[i] = r * w * dz[i] - r3 * u[i] * dot;
        }
        storev<EPL>(dr + which * HD + h * D + lane * EPL, du);
      }
      float g[EPL];
      loadv<EPL>(dv + irow + h * D + lane * EPL, g);
      storev<EPL>(dr + 2 * HD + h * D + lane * EPL, g);
    }
  }
#pragma unroll
  for (int m = 0; m < 2; ++m)
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      if (acc[m][0][i] != 0.f) atomicAdd(dqw + m * D + lane * EPL + i, acc[m][0][i]);
      if (acc[m][1][i] != 0.f) atomicAdd(dkw + m * D + lane * EPL + i, acc[m][1][i]);
    }
}

int grid_for(int L) {
  int blocks = (L + 7) / 8;
  return blocks < 148 * 8 ? (blocks > 0 ? blocks : 1) : 148 * 8;
}

}  // namespace

const char* launch_qkv_post_fwd(const void* raw, const float* qw, const float* kw, const float* cos_t,
                                const float* sin_t, const int* itc, int nv, int na, int L, int H, int D, float eps,
                                void* q, void* k, void* v, cudaStream_t s, const uint64_t* peer_q,
                                const uint64_t* peer_k, const uint64_t* peer_v, int cp, int rank) {
  auto R = (const __nv_bfloat16*)raw;
  auto Q = (__nv_bfloat16*)q;
  auto K = (__nv_bfloat16*)k;
  auto V = (__nv_bfloat16*)v;
  const bool scatter = peer_q != nullptr;
  if (scatter && (peer_k == nullptr || peer_v == nullptr || cp < 1 || H % cp || rank < 0 || rank >= cp))
    return "qkv_post: bad Ulysses scatter arguments";
  const HeadScatter hs{peer_q, peer_k, peer_v, scatter ? cp : 1, scatter ? rank : 0, scatter ? H / cp : H};
  if (D == 128)
    qkv_post_fwd_kernel<4><<<grid_for(L), 256, 0, s>>>(R, qw, kw, cos_t, sin_t, itc, nv, na, L, H, eps, Q, K, V, hs);
  else if (D == 64)
    qkv_post_fwd_kernel<2><<<grid_for(L), 256, 0, s>>>(R, qw, kw, cos_t, sin_t, itc, nv, na, L, H, eps, Q, K, V, hs);
  else
    return "qkv_post: head_dim must be 64 or 128";
  return cudaGetLastError() == cudaSuccess ? nullptr : "qkv_post: launch failed";
}

const char* launch_qkv_post_bwd(const void* dq, const void* dk, const void* dv, const void* raw, const float* qw,
                                const float* kw, const float* cos_t, const float* sin_t, const int* itc, int nv,
                                int na, int L, int H, int D, float eps, void* draw, float* dqw, float* dkw,
                                cudaStream_t s) {
  auto cb = [](const void* p) { return (const __nv_bfloat16*)p; };
  if (D == 128)
    qkv_post_bwd_kernel<4><<<grid_for(L), 256, 0, s>>>(cb(dq), cb(dk), cb(dv), cb(raw), qw, kw, cos_t, sin_t, itc, nv,
                                                       na, L, H, eps, (__nv_bfloat16*)draw, dqw, dkw);
  else if (D == 64)
    qkv_post_bwd_kernel<2><<<grid_for(L), 256, 0, s>>>(cb(dq), cb(dk), cb(dv), cb(raw), qw, kw, cos_t, sin_t, itc, nv,
                                                       na, L, H, eps, (__nv_bfloat16*)draw, dqw, dkw);
  else
    return "qkv_post: head_dim must be 64 or 128";
  return nullptr;
}

// Index errors recorded by the bounds-checked debug build in this file's kernels (0 otherwise).
int qkv_bounds_error(bool reset) {
#ifdef PAN_DEBUG_BOUNDS
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_bounds_error, sizeof(int));
  if (reset) {
    int z = 0;
    cudaMemcpyToSymbol(g_bounds_error, &z, sizeof(int));
  }
  return v;
#else
  (void)reset;
  return 0;
#endif
}

}  // namespace pan
