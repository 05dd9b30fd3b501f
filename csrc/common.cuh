// Shared device helpers for the pan2_b200 sm_100a kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace pan {

// Bounds-checked debug build (compile with -DPAN_DEBUG_BOUNDS, e.g. PAN_DEBUG_BOUNDS=1 python setup.py
// build_ext --inplace): PAN_IDX(i, n, code) checks a data-driven index against its bound, records
// `code` in the device error flag read by error_flag() when it is out of range, and substitutes 0 so
// the access stays in bounds.  In the normal build the macro is the bare index expression, so the
// production kernels compile exactly as written.
#ifdef PAN_DEBUG_BOUNDS
static __device__ int g_bounds_error = 0;  // one per translation unit; each file exposes a reader
__device__ __forceinline__ int pan_checked_index(int i, int n, int code) {
  if (i < 0 || i >= n) {
    atomicCAS(&g_bounds_error, 0, code);
    return 0;
  }
  return i;
}
#define PAN_IDX(i, n, code) ::pan::pan_checked_index((i), (n), (code))
#else
#define PAN_IDX(i, n, code) (i)
#endif

// 8 x bf16 = 16 bytes, the unit of every vectorised row access.
struct __align__(16) bf16x8 {
  __nv_bfloat162 h[4];
};

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&v)[8]) {
  bf16x8 r = *reinterpret_cast<const bf16x8*>(p);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __bfloat1622float2(r.h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

__device__ __forceinline__ void store8(__nv_bfloat16* p, const float (&v)[8]) {
  bf16x8 r;
#pragma unroll
  for (int i = 0; i < 4; ++i) r.h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<bf16x8*>(p) = r;
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Round-trip through bf16 (the value a consumer reading the stored tensor sees).
__device__ __forceinline__ void round8(float (&v)[8]) {
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __bfloat162float(__float2bfloat16_rn(v[i]));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Segment of `row` given boundaries b[0..n_seg] (b[0] == 0); -1 when outside [b[0], b[n_seg]).
__device__ __forceinline__ int find_segment(const int* b, int n_seg, int row) {
  if (row < b[0] || row >= b[n_seg]) return -1;
  int s = 0;
  while (s + 1 < n_seg && row >= b[s + 1]) ++s;
  return s;
}

}  // namespace pan
