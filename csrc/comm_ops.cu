// Collectives over NVLink peer memory (symmetric buffers mapped into every rank of a node).
//
//   symm_barrier   every rank stores an epoch into each peer's signal slot and waits (bounded)
//                  until all peers' epochs for it are at least that epoch;
//   peer_gather    the FSDP parameter all-gather fused with the shard -> natural-layout unpack:
//                  each rank pulls every peer's bf16 shard rows straight into its full weights;
//   peer_reduce    the gradient reduce-scatter fused with the bf16 -> fp32 cast and the scale:
//                  each rank sums its own rows of every peer's bf16 gradient in fp32;
//   peer_gemv      the parameter all-gather fused into a skinny projection (the AdaLN modulation,
//                  k <= 8 rows): y[j, n] = sum_c a[j, c] W[n, c] + bias[n], every weight row read
//                  once, straight from the peer that owns it, and never written locally.
// Segments describe contiguous runs (element offsets): for peer_gather `src` is an offset in the
// peer's buffer and `dst` in the local output; for peer_reduce `src` is an offset in every peer's
// gradient buffer and `dst` in the local fp32 shard.  All loads / stores are 16-byte vectors when
// the run is aligned, elements otherwise.  Spin-waits give up after 4 s, record an error code and
// return, so a missing peer cannot hang the GPU.
#include <stdint.h>

#include "common.cuh"
#include "launchers.h"

namespace pan {
namespace {

__device__ int g_comm_error = 0;

struct Seg {
  long long src, dst, n;
};

__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
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

// one block; thread k < world signals peer k and waits for peer k
__global__ void symm_barrier_kernel(const uint64_t* __restrict__ pads, int rank, int world, uint32_t epoch,
                                    int channel, uint64_t limit_ns) {
  const int k = threadIdx.x;
  if (k >= world) return;
  uint32_t* peer_pad = reinterpret_cast<uint32_t*>(pads[k]) + channel * 64;
  st_release_sys(peer_pad + rank, epoch);
  const uint32_t* mine = reinterpret_cast<const uint32_t*>(pads[rank]) + channel * 64 + k;
  const uint64_t t0 = now_ns();
  while ((int)(ld_acquire_sys(mine) - epoch) < 0) {
    if (now_ns() - t0 > limit_ns) {
      atomicCAS(&g_comm_error, 0, 100 + k);
      return;
    }
  }
}

__device__ __forceinline__ int find_seg(const long long* prefix, int n_seg, long long i) {
  int lo = 0, hi = n_seg - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (prefix[mid] <= i) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

// out[dst + j] = peer_{seg.peer}[src + j]; segments carry their peer in the high bits of `n`'s
// companion array (peer index per segment)
__global__ void peer_gather_kernel(const uint64_t* __restrict__ peers, const Seg* __restrict__ segs,
                                   const int* __restrict__ seg_peer, const long long* __restrict__ prefix,
                                   int n_seg, long long total, __nv_bfloat16* __restrict__ out) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  // 8-element units: prefix counts units per segment when the segment is aligned, elements otherwise
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int s = find_seg(prefix, n_seg, i);
    const Seg g = segs[s];
    const long long j = i - prefix[s];
    const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(peers[seg_peer[s]]);
    const bool vec = ((g.src | g.dst | g.n) & 7) == 0;
    if (vec) {
      *reinterpret_cast<uint4*>(out + g.dst + 8 * j) = *reinterpret_cast<const uint4*>(src + g.src + 8 * j);
    } else {
      out[g.dst + j] = src[g.src + j];
    }
  }
}

template <int MAXW>
__global__ void peer_reduce_kernel(const uint64_t* __restrict__ peers, int world, const Seg* __restrict__ segs,
                                   const long long* __restrict__ prefix, int n_seg, long long total, float scale,
                                   float* __restrict__ out) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int s = find_seg(prefix, n_seg, i);
    const Seg g = segs[s];
    const long long j = i - prefix[s];
    const bool vec = ((g.src | g.dst | g.n) & 7) == 0;
    if (vec) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
      for (int k = 0; k < world; ++k) {
        float v[8];
        load8(reinterpret_cast<const __nv_bfloat16*>(peers[k]) + g.src + 8 * j, v);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] += v[e];
      }
      float* o = out + g.dst + 8 * j;
      *reinterpret_cast<float4*>(o) = make_float4(acc[0] * scale, acc[1] * scale, acc[2] * scale, acc[3] * scale);
      *reinterpret_cast<float4*>(o + 4) = make_float4(acc[4] * scale, acc[5] * scale, acc[6] * scale, acc[7] * scale);
    } else {
      float acc = 0.f;
      for (int k = 0; k < world; ++k)
        acc += __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(peers[k])[g.src + j]);
      out[g.dst + j] = acc * scale;
    }
  }
}

// ---------------------------------------------------------------------------------------------
// peer_gemv: W [N, K] is row-sharded over the ranks (rank r holds rows [r*R, min(N, (r+1)*R)) at
// element offset w_off of its buffer); a [k, K] (k <= 8) is staged in shared memory once per CTA.
// One warp owns one output row at a time: its 32 lanes stream the row's 16-byte vectors from the
// owner over NVLink (PV loads in flight per lane before any math), multiply them into k fp32
// accumulators and reduce across the warp.  Memory-bound by design; CUDA cores are ample for
// k <= 8 (the tensor cores' smallest tile is 64 rows).
constexpr int GEMV_WARPS = 8;
constexpr int GEMV_PV = 4;  // 16-byte W vectors in flight per lane

template <int KR>
__global__ void __launch_bounds__(GEMV_WARPS * 32)
peer_gemv_kernel(const uint64_t* __restrict__ peers, long long w_off, int rows_per_rank, int N, int K,
                 const __nv_bfloat16* __restrict__ a, const __nv_bfloat16* __restrict__ bias,
                 __nv_bfloat16* __restrict__ y) {
  extern __shared__ uint4 a_s[];  // KR rows x K/8 vectors
  const int kv = K >> 3;
  for (int i = threadIdx.x; i < KR * kv; i += blockDim.x) a_s[i] = reinterpret_cast<const uint4*>(a)[i];
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int warp = blockIdx.x * GEMV_WARPS + (threadIdx.x >> 5);
  const int n_warps = gridDim.x * GEMV_WARPS;
  for (int n = warp; n < N; n += n_warps) {
    const int r = n / rows_per_rank;
    const uint4* w = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(peers[r]) + w_off +
                                                    (long long)(n - r * rows_per_rank) * K);
    float acc[KR];
#pragma unroll
    for (int j = 0; j < KR; ++j) acc[j] = 0.f;
    for (int c0 = lane; c0 < kv; c0 += 32 * GEMV_PV) {
      uint4 wv[GEMV_PV];
#pragma unroll
      for (int u = 0; u < GEMV_PV; ++u) {
        const int c = c0 + 32 * u;
        wv[u] = c < kv ? w[c] : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < GEMV_PV; ++u) {
        const int c = c0 + 32 * u;
        if (c >= kv) break;
        const __nv_bfloat162* wh = reinterpret_cast<const __nv_bfloat162*>(&wv[u]);
        float2 wf[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) wf[e] = __bfloat1622float2(wh[e]);
#pragma unroll
        for (int j = 0; j < KR; ++j) {
          const uint4 av = a_s[j * kv + c];
          const __nv_bfloat162* ah = reinterpret_cast<const __nv_bfloat162*>(&av);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 af = __bfloat1622float2(ah[e]);
            acc[j] = fmaf(af.x, wf[e].x, acc[j]);
            acc[j] = fmaf(af.y, wf[e].y, acc[j]);
          }
        }
      }
    }
#pragma unroll
    for (int j = 0; j < KR; ++j) acc[j] = warp_sum(acc[j]);
    if (lane < KR) {
      float v = 0.f;
#pragma unroll
      for (int j = 0; j < KR; ++j)
        if (j == lane) v = acc[j];
      if (bias != nullptr) v += __bfloat162float(bias[n]);
      y[(long long)lane * N + n] = __float2bfloat16_rn(v);
    }
  }
}

int grid_for(long long total) {
  long long b = (total + 255) / 256;
  return (int)(b < 148 * 8 ? (b < 1 ? 1 : b) : 148 * 8);
}

}  // namespace

const char* launch_symm_barrier(const uint64_t* pads, int rank, int world, uint32_t epoch, int channel,
                                int timeout_ms, cudaStream_t s) {
  if (world > 64) return "symm_barrier: at most 64 ranks";
  symm_barrier_kernel<<<1, 64, 0, s>>>(pads, rank, world, epoch, channel, (uint64_t)timeout_ms * 1000000ull);
  return cudaGetLastError() == cudaSuccess ? nullptr : "symm_barrier: launch failed";
}

const char* launch_peer_gather(const uint64_t* peers, const void* segs, const int* seg_peer, const long long* prefix,
                               int n_seg, long long total, void* out, cudaStream_t s) {
  if (total <= 0) return nullptr;
  peer_gather_kernel<<<grid_for(total), 256, 0, s>>>(peers, reinterpret_cast<const Seg*>(segs), seg_peer, prefix,
                                                     n_seg, total, reinterpret_cast<__nv_bfloat16*>(out));
  return cudaGetLastError() == cudaSuccess ? nullptr : "peer_gather: launch failed";
}

const char* launch_peer_reduce(const uint64_t* peers, int world, const void* segs, const long long* prefix, int n_seg,
                               long long total, float scale, float* out, cudaStream_t s) {
  if (total <= 0) return nullptr;
  peer_reduce_kernel<64><<<grid_for(total), 256, 0, s>>>(peers, world, reinterpret_cast<const Seg*>(segs), prefix,
                                                         n_seg, total, scale, out);
  return cudaGetLastError() == cudaSuccess ? nullptr : "peer_reduce: launch failed";
}

const char* launch_peer_gemv(const uint64_t* peers, long long w_off, int rows_per_rank, int N, int K, int k,
                             const void* a, const void* bias, void* y, int n_sms, cudaStream_t s) {
  if (k < 1 || k > 8) return "peer_gemv: 1 <= k <= 8 rows";
  if (K % 8 != 0 || (w_off & 7) != 0) return "peer_gemv: K and the weight offset must be multiples of 8 elements";
  if (N <= 0) return nullptr;
  const size_t smem = (size_t)k * K * 2;
  if (smem > 200 * 1024) return "peer_gemv: k x K activations exceed shared memory";
  const int warps_needed = N;
  int ctas = (warps_needed + GEMV_WARPS - 1) / GEMV_WARPS;
  const int cap = n_sms * (smem > 96 * 1024 ? 1 : 2);
  if (ctas > cap) ctas = cap;
  const __nv_bfloat16* A = reinterpret_cast<const __nv_bfloat16*>(a);
  const __nv_bfloat16* B = reinterpret_cast<const __nv_bfloat16*>(bias);
  __nv_bfloat16* Y = reinterpret_cast<__nv_bfloat16*>(y);
  auto go = [&](auto kern) -> const char* {
    if (smem > 48 * 1024 && cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
                                cudaSuccess)
      return "peer_gemv: shared memory attribute refused";
    kern<<<ctas, GEMV_WARPS * 32, smem, s>>>(peers, w_off, rows_per_rank, N, K, A, B, Y);
    return cudaGetLastError() == cudaSuccess ? nullptr : "peer_gemv: launch failed";
  };
  switch (k) {
    case 1: return go(peer_gemv_kernel<1>);
    case 2: return go(peer_gemv_kernel<2>);
    case 3: return go(peer_gemv_kernel<3>);
    case 4: return go(peer_gemv_kernel<4>);
    case 5: return go(peer_gemv_kernel<5>);
    case 6: return go(peer_gemv_kernel<6>);
    case 7: return go(peer_gemv_kernel<7>);
    default: return go(peer_gemv_kernel<8>);
  }
}

int comm_error_flag(bool reset) {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_comm_error, sizeof(int));
  if (reset) {
    int z = 0;
    cudaMemcpyToSymbol(g_comm_error, &z, sizeof(int));
  }
  return v;
}

}  // namespace pan
