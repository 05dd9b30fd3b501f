// Packed-sequence elementwise kernels (sm_100a): LN-modulate, gate+residual with LayerNorm
// statistics, the [video | text + type | pad] concat, the video-row MSE, segment sums and row
// gathers.  All operate on bf16 [L, C] row-major activations with C % 256 == 0; segment
// boundaries are a small int32 device array.
//
// Semantics follow the reference's Triton kernels (pan/models/transformers/modules/
// triton_kernels.py:69-1073): ln_stats = (sum_c x, sum_c x^2) fp32 per row, LayerNorm eps 1e-6,
// mean = s0 / C, var = s1 / C - mean^2.
//
// Layout of the work: one warp owns one row (memory-bound, no shared-memory reductions); lanes
// stride the row in 16-byte vectors so a warp reads 512 contiguous bytes per step.  The LN-modulate
// forward instead gives each CTA a 2048-column slab and a run of rows (see its kernel).  Column
// reductions over rows (modulation/gate gradients, bias sums) use 256-thread CTAs that own 2048
// columns and a chunk of rows and flush fp32 partials with atomics at segment ends.
#include "common.cuh"
#include "launchers.h"

namespace pan {
namespace {

constexpr float kLnEps = 1e-6f;
constexpr int kMaxSeg = 64;

__device__ __forceinline__ void load_bounds(const int* __restrict__ bounds, int n_seg, int* sb) {
  for (int i = threadIdx.x; i <= n_seg; i += blockDim.x) sb[i] = bounds[i];
  __syncthreads();
}

// y = LN(x) * (1 + scale[seg]) + shift[seg]; padding rows -> 0.
// A CTA owns a 2048-column slab (8 columns per thread, one 16-byte vector) and a run of
// consecutive rows.  Consecutive rows almost always share a segment, so each thread keeps its
// columns of shift and (1 + scale) in registers and reloads them only when the segment changes;
// per row a thread then reads 16 bytes of x and writes 16 bytes of y (plus the row's two
// statistics, one broadcast load per warp), which keeps the kernel on DRAM bandwidth rather than on
// L1 re-reads of the modulation rows.  Rows are processed ROWS at a time so several loads are in
// flight per thread.
constexpr int LNM_COLS = 2048;
constexpr int LNM_ROWS = 8;       // rows in flight per thread (raw 16-byte vectors, 128 bytes)
constexpr int LNM_CTAS_PER_SM = 3;
__global__ void __launch_bounds__(256, LNM_CTAS_PER_SM) ln_modulate_fwd_kernel(
    const __nv_bfloat16* __restrict__ x, const float* __restrict__ stats, const __nv_bfloat16* __restrict__ shift,
    const __nv_bfloat16* __restrict__ scale, const int* __restrict__ bounds, int n_seg, int L, int C,
    int rows_per_cta, __nv_bfloat16* __restrict__ y) {
  __shared__ int sb[kMaxSeg + 1];
  load_bounds(bounds, n_seg, sb);
  const int c = blockIdx.x * LNM_COLS + threadIdx.x * 8;
  if (c >= C) return;
  const int r0 = blockIdx.y * rows_per_cta;
  const int r1 = min(L, r0 + rows_per_cta);
  int seg = -2, seg_end = -1;  // segment of the cached modulation columns; first row past it
  float hv[8], sv1[8];
  const float inv_c = 1.f / C;
  for (int row = r0; row < r1; row += LNM_ROWS) {
    uint4 raw[LNM_ROWS];
#pragma unroll
    for (int k = 0; k < LNM_ROWS; ++k)
      raw[k] = row + k < r1 ? *reinterpret_cast<const uint4*>(x + (size_t)(row + k) * C + c) : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int k = 0; k < LNM_ROWS; ++k) {
      const int r = row + k;
      if (r >= r1) break;
      if (r >= seg_end) {
        seg = find_segment(sb, n_seg, r);
        if (seg >= 0) {
          seg_end = sb[seg + 1];
          load8(shift + (size_t)seg * C + c, hv);
          load8(scale + (size_t)seg * C + c, sv1);
#pragma unroll
          for (int i = 0; i < 8; ++i) sv1[i] += 1.f;
        } else {
          seg_end = r < sb[0] ? sb[0] : L;  // the next row that can be inside a segment
        }
      }
      float o[8];
      if (seg < 0) {
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = 0.f;
      } else {
        const float2 st = *reinterpret_cast<const float2*>(stats + 2 * (size_t)r);
        const float mean = st.x * inv_c;
        const float rstd = rsqrtf(fmaxf(st.y * inv_c - mean * mean, 0.f) + kLnEps);
        const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw[k]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 xv = __bfloat1622float2(h2[i]);
          o[2 * i] = (xv.x - mean) * rstd * sv1[2 * i] + hv[2 * i];
          o[2 * i + 1] = (xv.y - mean) * rstd * sv1[2 * i + 1] + hv[2 * i + 1];
        }
      }
      store8(y + (size_t)r * C + c, o);
    }
  }
}

// dx = rstd * (dn - mean(dn) - n * mean(dn * n)),  dn = g * (1 + scale[seg]).
__global__ void ln_modulate_bwd_dx_kernel(const __nv_bfloat16* __restrict__ g, const __nv_bfloat16* __restrict__ x,
                                          const float* __restrict__ stats, const __nv_bfloat16* __restrict__ scale,
                                          const int* __restrict__ bounds, int n_seg, int L, int C,
                                          __nv_bfloat16* __restrict__ dx) {
  __shared__ int sb[kMaxSeg + 1];
  load_bounds(bounds, n_seg, sb);
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < L; row += gridDim.x * warps) {
    const int seg = find_segment(sb, n_seg, row);
    __nv_bfloat16* dr = dx + (size_t)row * C;
    if (seg < 0) {
      float z[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int c = lane * 8; c < C; c += 256) store8(dr + c, z);
      continue;
    }
    const float s0 = stats[2 * row], s1 = stats[2 * row + 1];
    const float mean = s0 / C;
    const float rstd = rsqrtf(fmaxf(s1 / C - mean * mean, 0.f) + kLnEps);
    const __nv_bfloat16* gr = g + (size_t)row * C;
    const __nv_bfloat16* xr = x + (size_t)row * C;
    const __nv_bfloat16* sc = scale + (size_t)seg * C;
    float a = 0.f, b = 0.f;
    for (int c = lane * 8; c < C; c += 256) {
      float gv[8], xv[8], sv[8];
      load8(gr + c, gv);
      load8(xr + c, xv);
      load8(sc + c, sv);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float dn = gv[i] * (1.f + sv[i]);
        const float n = (xv[i] - mean) * rstd;
        a += dn;
        b += dn * n;
      }
    }
    a = warp_sum(a) / C;
    b = warp_sum(b) / C;
    for (int c = lane * 8; c < C; c += 256) {
      float gv[8], xv[8], sv[8], o[8];
      load8(gr + c, gv);
      load8(xr + c, xv);
      load8(sc + c, sv);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float dn = gv[i] * (1.f + sv[i]);
        const float n = (xv[i] - mean) * rstd;
        o[i] = rstd * (dn - a - n * b);
      }
      store8(dr + c, o);
    }
  }
}

// Column reductions over the rows of each segment.
//   mode 0: out0[s, c] += sum g                         (segment / column sums)
//   mode 1: out0 += sum g, out1 += sum g * LN(x)        (ln-modulate dshift, dscale)
//   mode 2: out0 += sum g * y                           (gate gradient)
// Grid: x = column tiles of 2048, y = row chunks.  Every CTA walks its rows in order and flushes
// its register partials with atomics when the segment changes and at the end.
template <int MODE>
__global__ void column_reduce_kernel(const __nv_bfloat16* __restrict__ g, const __nv_bfloat16* __restrict__ x,
                                     const float* __restrict__ stats, const int* __restrict__ bounds, int n_seg,
                                     int C, int rows_per_chunk, float* __restrict__ out0,
                                     float* __restrict__ out1) {
  __shared__ int sb[kMaxSeg + 1];
  load_bounds(bounds, n_seg, sb);
  const int c = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  const int r_begin = max(blockIdx.y * rows_per_chunk, sb[0]);
  const int r_end = min((int)(blockIdx.y + 1) * rows_per_chunk, sb[n_seg]);
  if (c >= C || r_begin >= r_end) return;
  float acc0[8], acc1[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc0[i] = acc1[i] = 0.f;
  int seg = find_segment(sb, n_seg, r_begin);
  int seg_end = sb[seg + 1];
  auto flush = [&](int s) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      atomicAdd(out0 + (size_t)s * C + c + i, acc0[i]);
      if (MODE == 1) atomicAdd(out1 + (size_t)s * C + c + i, acc1[i]);
      acc0[i] = acc1[i] = 0.f;
    }
  };
  for (int r = r_begin; r < r_end; ++r) {
    if (r >= seg_end) {
      flush(seg);
      while (r >= sb[seg + 1]) ++seg;
      seg_end = sb[seg + 1];
    }
    float gv[8];
    load8(g + (size_t)r * C + c, gv);
    if (MODE == 0) {
#pragma unroll
      for (int i = 0; i < 8; ++i) acc0[i] += gv[i];
    } else if (MODE == 1) {
      float xv[8];
      load8(x + (size_t)r * C + c, xv);
      const float mean = stats[2 * r] / C;
      const float rstd = rsqrtf(fmaxf(stats[2 * r + 1] / C - mean * mean, 0.f) + kLnEps);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        acc0[i] += gv[i];
        acc1[i] += gv[i] * (xv[i] - mean) * rstd;
      }
    } else {
      float xv[8];
      load8(x + (size_t)r * C + c, xv);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc0[i] += gv[i] * xv[i];
    }
  }
  flush(seg);
}

// out = y * gate[seg] + res (padding rows: out = res), stats = (sum out, sum out^2) of the
// bf16-rounded output (zero on padding rows).
__global__ void gate_residual_fwd_kernel(const __nv_bfloat16* __restrict__ y, const __nv_bfloat16* __restrict__ gate,
                                         const __nv_bfloat16* __restrict__ res, const int* __restrict__ bounds,
                                         int n_seg, int L, int C, __nv_bfloat16* __restrict__ out,
                                         float* __restrict__ stats) {
  __shared__ int sb[kMaxSeg + 1];
  load_bounds(bounds, n_seg, sb);
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < L; row += gridDim.x * warps) {
    const int seg = find_segment(sb, n_seg, row);
    const __nv_bfloat16* yr = y + (size_t)row * C;
    const __nv_bfloat16* rr = res + (size_t)row * C;
    __nv_bfloat16* orow = out + (size_t)row * C;
    float s0 = 0.f, s1 = 0.f;
    for (int c = lane * 8; c < C; c += 256) {
      float rv[8], o[8];
      load8(rr + c, rv);
      if (seg >= 0) {
        float yv[8], gv[8];
        load8(yr + c, yv);
        load8(gate + (size_t)seg * C + c, gv);
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = yv[i] * gv[i] + rv[i];
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = rv[i];
      }
      round8(o);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        s0 += o[i];
        s1 += o[i] * o[i];
      }
      store8(orow + c, o);
    }
    s0 = warp_sum(s0);
    s1 = warp_sum(s1);
    if (lane == 0) {
      stats[2 * row] = seg >= 0 ? s0 : 0.f;
      stats[2 * row + 1] = seg >= 0 ? s1 : 0.f;
    }
  }
}

// dy = g * gate[seg] (padding rows 0).
__global__ void gate_bwd_dy_kernel(const __nv_bfloat16* __restrict__ g, const __nv_bfloat16* __restrict__ gate,
                                   const int* __restrict__ bounds, int n_seg, int L, int C,
                                   __nv_bfloat16* __restrict__ dy) {
  __shared__ int sb[kMaxSeg + 1];
  load_bounds(bounds, n_seg, sb);
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < L; row += gridDim.x * warps) {
    const int seg = find_segment(sb, n_seg, row);
    __nv_bfloat16* dr = dy + (size_t)row * C;
    for (int c = lane * 8; c < C; c += 256) {
      float o[8];
      if (seg >= 0) {
        float gv[8], tv[8];
        load8(g + (size_t)row * C + c, gv);
        load8(gate + (size_t)seg * C + c, tv);
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = gv[i] * tv[i];
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = 0.f;
      }
      store8(dr + c, o);
    }
  }
}

// [video | text + ttv | zero pad] with stats of the stored rows.
__global__ void concat_fwd_kernel(const __nv_bfloat16* __restrict__ vid, const __nv_bfloat16* __restrict__ txt,
                                  const __nv_bfloat16* __restrict__ ttv, int nv, int nt, int L, int C,
                                  __nv_bfloat16* __restrict__ out, float* __restrict__ stats) {
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < L; row += gridDim.x * warps) {
    __nv_bfloat16* orow = out + (size_t)row * C;
    float s0 = 0.f, s1 = 0.f;
    for (int c = lane * 8; c < C; c += 256) {
      float o[8];
      if (row < nv) {
        load8(vid + (size_t)row * C + c, o);
      } else if (row < nv + nt) {
        load8(txt + (size_t)(row - nv) * C + c, o);
        if (ttv != nullptr) {
          float t[8];
          load8(ttv + c, t);
#pragma unroll
          for (int i = 0; i < 8; ++i) o[i] += t[i];
        }
        round8(o);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = 0.f;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        s0 += o[i];
        s1 += o[i] * o[i];
      }
      store8(orow + c, o);
    }
    s0 = warp_sum(s0);
    s1 = warp_sum(s1);
    if (lane == 0) {
      stats[2 * row] = s0;
      stats[2 * row + 1] = s1;
    }
  }
}

// Per-CTA partial sums of (pred - target)^2 over the first nv rows; deterministic 2-stage reduce.
__global__ void mse_partial_kernel(const __nv_bfloat16* __restrict__ pred, const __nv_bfloat16* __restrict__ tgt,
                                   size_t n, float* __restrict__ partial) {
  float acc = 0.f;
  const size_t stride = (size_t)gridDim.x * blockDim.x * 8;
  for (size_t i = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) * 8; i < n; i += stride) {
    float p[8], t[8];
    load8(pred + i, p);
    load8(tgt + i, t);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float d = p[k] - t[k];
      acc += d * d;
    }
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

__global__ void mse_final_kernel(const float* __restrict__ partial, int n_part, float count, float* __restrict__ out) {
  float acc = 0.f;
  for (int i = threadIdx.x; i < n_part; i += blockDim.x) acc += partial[i];
  acc = warp_sum(acc);
  __shared__ float ws[32];
  if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? ws[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) {
      out[0] = v;
      out[1] = count;
    }
  }
}

// dpred = 2 (pred - target) * gsum[0] on the first n elements; zero beyond (up to total).
__global__ void mse_bwd_kernel(const __nv_bfloat16* __restrict__ pred, const __nv_bfloat16* __restrict__ tgt,
                               const float* __restrict__ gsum, size_t n, size_t total,
                               __nv_bfloat16* __restrict__ dpred) {
  const float s = 2.f * gsum[0];
  const size_t stride = (size_t)gridDim.x * blockDim.x * 8;
  for (size_t i = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) * 8; i < total; i += stride) {
    float o[8];
    if (i < n) {
      float p[8], t[8];
      load8(pred + i, p);
      load8(tgt + i, t);
#pragma unroll
      for (int k = 0; k < 8; ++k) o[k] = s * (p[k] - t[k]);
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) o[k] = 0.f;
    }
    store8(dpred + i, o);
  }
}

// out[i, :] = x[idx[i], :] for rows of `row_bytes` bytes (multiple of 16).
__global__ void gather_rows_kernel(const uint4* __restrict__ x, const int* __restrict__ idx, int rows, int vec_per_row,
                                   uint4* __restrict__ out) {
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  for (int r = blockIdx.x * warps + (threadIdx.x >> 5); r < rows; r += gridDim.x * warps) {
    const uint4* src = x + (size_t)idx[r] * vec_per_row;
    uint4* dst = out + (size_t)r * vec_per_row;
    for (int v = lane; v < vec_per_row; v += 32) dst[v] = src[v];
  }
}

int row_grid(int L) {
  const int warps = 8;
  int blocks = (L + warps - 1) / warps;
  return blocks < 148 * 16 ? (blocks > 0 ? blocks : 1) : 148 * 16;
}

template <int MODE>
void column_reduce(const void* g, const void* x, const float* stats, const int* bounds, int n_seg, int L, int C,
                   float* out0, float* out1, cudaStream_t s) {
  const int rows_per_chunk = 128;
  dim3 grid((C + 2047) / 2048, (L + rows_per_chunk - 1) / rows_per_chunk);
  if (grid.y == 0) return;
  column_reduce_kernel<MODE><<<grid, 256, 0, s>>>((const __nv_bfloat16*)g, (const __nv_bfloat16*)x, stats, bounds,
                                                  n_seg, C, rows_per_chunk, out0, out1);
}

}  // namespace

#define BF(p) reinterpret_cast<__nv_bfloat16*>(p)
#define CBF(p) reinterpret_cast<const __nv_bfloat16*>(p)

void launch_ln_modulate_fwd(const void* x, const float* stats, const void* shift, const void* scale,
                            const int* bounds, int n_seg, int L, int C, void* y, cudaStream_t s) {
  if (L <= 0) return;
  const int slabs = (C + LNM_COLS - 1) / LNM_COLS;
  // one wave: LNM_CTAS_PER_SM CTAs per SM in total, rows split evenly (a multiple of the unroll)
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  }
  const int chunks = (sms * LNM_CTAS_PER_SM + slabs - 1) / slabs;
  int rows = (L + chunks - 1) / chunks;
  rows = (rows + LNM_ROWS - 1) / LNM_ROWS * LNM_ROWS;
  const dim3 grid(slabs, (L + rows - 1) / rows);
  ln_modulate_fwd_kernel<<<grid, 256, 0, s>>>(CBF(x), stats, CBF(shift), CBF(scale), bounds, n_seg, L, C, rows,
                                              BF(y));
}

void launch_ln_modulate_bwd(const void* g, const void* x, const float* stats, const void* scale, const int* bounds,
                            int n_seg, int L, int C, void* dx, float* dshift, float* dscale, cudaStream_t s) {
  ln_modulate_bwd_dx_kernel<<<row_grid(L), 256, 0, s>>>(CBF(g), CBF(x), stats, CBF(scale), bounds, n_seg, L, C,
                                                        BF(dx));
  column_reduce<1>(g, x, stats, bounds, n_seg, L, C, dshift, dscale, s);
}

void launch_gate_residual_fwd(const void* y, const void* gate, const void* res, const int* bounds, int n_seg, int L,
                              int C, void* out, float* stats, cudaStream_t s) {
  gate_residual_fwd_kernel<<<row_grid(L), 256, 0, s>>>(CBF(y), CBF(gate), CBF(res), bounds, n_seg, L, C, BF(out),
                                                       stats);
}

void launch_gate_bwd(const void* g, const void* y, const void* gate, const int* bounds, int n_seg, int L, int C,
                     void* dy, float* dgate, cudaStream_t s) {
  gate_bwd_dy_kernel<<<row_grid(L), 256, 0, s>>>(CBF(g), CBF(gate), bounds, n_seg, L, C, BF(dy));
  column_reduce<2>(g, y, nullptr, bounds, n_seg, L, C, dgate, nullptr, s);
}

void launch_concat_fwd(const void* vid, const void* txt, const void* ttv, int nv, int nt, int L, int C, void* out,
                       float* stats, cudaStream_t s) {
  concat_fwd_kernel<<<row_grid(L), 256, 0, s>>>(CBF(vid), CBF(txt), CBF(ttv), nv, nt, L, C, BF(out), stats);
}

void launch_segment_sum(const void* x, const int* bounds, int n_seg, int L, int C, float* out, cudaStream_t s) {
  column_reduce<0>(x, nullptr, nullptr, bounds, n_seg, L, C, out, nullptr, s);
}

void launch_mse_fwd(const void* pred, const void* tgt, size_t n, float* partial, int n_part, float* out,
                    cudaStream_t s) {
  mse_partial_kernel<<<n_part, 256, 0, s>>>(CBF(pred), CBF(tgt), n, partial);
  mse_final_kernel<<<1, 1024, 0, s>>>(partial, n_part, (float)n, out);
}

void launch_mse_bwd(const void* pred, const void* tgt, const float* gsum, size_t n, size_t total, void* dpred,
                    cudaStream_t s) {
  mse_bwd_kernel<<<148 * 8, 256, 0, s>>>(CBF(pred), CBF(tgt), gsum, n, total, BF(dpred));
}

void launch_gather_rows(const void* x, const int* idx, int rows, int vec16_per_row, void* out, cudaStream_t s) {
  gather_rows_kernel<<<row_grid(rows), 256, 0, s>>>(reinterpret_cast<const uint4*>(x), idx, rows, vec16_per_row,
                                                    reinterpret_cast<uint4*>(out));
}

int packed_ops_error_flag(bool) { return 0; }

}  // namespace pan
