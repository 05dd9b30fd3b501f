// Allocation-free entry point for the flow-matching loss sums.
//
// This file has no counterpart in the reference project.  It exists for callers that cannot call
// cudaMalloc or any allocating library routine: runtimes and custom allocators that own every
// device allocation and forbid hidden ones, and C/C++ hosts that link this library without PyTorch
// and so have no caching allocator to borrow scratch space from.  The C declarations are in
// noalloc_mse.h:
//
//   int pan2_mse_sums_noalloc(const void* pred, const void* target, long long n, float* out,
//                             void* stream);
//
// computes, for bf16 `pred` and `target` of `n` elements each (device pointers, 16-byte aligned,
// n a multiple of 8), out[0] = sum((pred - target)^2) and out[1] = n (fp32, device pointer) -- the
// same values as the allocating `mse_fwd` binding.  The caller owns every input and output buffer.
//
// Scratch: the per-CTA partial sums live in the file-scope device array `g_mse_partials` below
// (kMaxPartials floats = 64 KB), which every GPU that loads this library keeps until the process
// exits.  One CTA handles 2048 elements, so n is limited to kMaxPartials * 2048 = 33,554,432
// elements; larger n is rejected with error code 2 and a message from pan2_noalloc_last_error().
//
// Host code cannot use `g_mse_partials` directly (on the host that name is only a stand-in for the
// device symbol), so the first call on each device looks up the array's device address with
// cudaGetSymbolAddress while that device is current, checks the result and caches it.  Make that
// first call on a device before any stream capture begins.
//
// Every call reuses the same array and each call overwrites every partial it later reads, so no
// clearing is needed; calls that run concurrently on the GPU (different streams, overlapping in
// time) race on the array and must be serialised by the caller.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <mutex>

#include "common.cuh"
#include "noalloc_mse.h"

constexpr int kMaxPartials = 16384;

// The scratch: per-CTA partial sums, shared by every call on a device.
static __device__ __align__(256) float g_mse_partials[kMaxPartials];

namespace {

constexpr int kTileElems = 2048;  // 256 threads x 8 elements
constexpr int kMaxDevices = 64;

// Device address of g_mse_partials per device, looked up once: read without the lock (acquire),
// written under it (release).
std::atomic<float*> g_partials_addr[kMaxDevices];
std::mutex g_setup_mutex;
thread_local const char* g_last_error = "no error";

__global__ void mse_tile_kernel(const __nv_bfloat16* __restrict__ pred, const __nv_bfloat16* __restrict__ tgt,
                                long long n, float* __restrict__ partial) {
  const long long i = (long long)blockIdx.x * kTileElems + threadIdx.x * 8;
  float acc = 0.f;
  if (i < n) {
    float p[8], t[8];
    pan::load8(pred + i, p);
    pan::load8(tgt + i, t);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float d = p[k] - t[k];
      acc += d * d;
    }
  }
  acc = pan::warp_sum(acc);
  __shared__ float ws[8];
  if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < 8 ? ws[threadIdx.x] : 0.f;
    v = pan::warp_sum(v);
    if (threadIdx.x == 0) partial[blockIdx.x] = v;
  }
}

__global__ void mse_final_kernel(const float* __restrict__ partial, int n_part, float count, float* __restrict__ out) {
  float acc = 0.f;
  for (int i = threadIdx.x; i < n_part; i += blockDim.x) acc += partial[i];
  acc = pan::warp_sum(acc);
  __shared__ float ws[32];
  if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? ws[threadIdx.x] : 0.f;
    v = pan::warp_sum(v);
    if (threadIdx.x == 0) {
      out[0] = v;
      out[1] = count;
    }
  }
}

}  // namespace

extern "C" {

// Message of the last failed call on this host thread.
const char* pan2_noalloc_last_error() { return g_last_error; }

// Returns 0 on success; 1 bad arguments, 2 n above the scratch limit, 3 CUDA error.
int pan2_mse_sums_noalloc(const void* pred, const void* target, long long n, float* out, void* stream) {
  if (pred == nullptr || target == nullptr || out == nullptr || n < 0 || n % 8 != 0 ||
      reinterpret_cast<uintptr_t>(pred) % 16 != 0 || reinterpret_cast<uintptr_t>(target) % 16 != 0) {
    g_last_error = "pan2_mse_sums_noalloc: null pointer, unaligned input or n not a multiple of 8";
    return 1;
  }
  const long long tiles = (n + kTileElems - 1) / kTileElems;
  if (tiles > kMaxPartials) {
    g_last_error = "pan2_mse_sums_noalloc: n exceeds the 33,554,432-element scratch limit";
    return 2;
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    g_last_error = "pan2_mse_sums_noalloc: no current CUDA device";
    return 3;
  }
  float* partials = g_partials_addr[dev].load(std::memory_order_acquire);
  if (partials == nullptr) {
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    partials = g_partials_addr[dev].load(std::memory_order_relaxed);
    if (partials == nullptr) {
      void* ptr = nullptr;
      if (cudaGetSymbolAddress(&ptr, g_mse_partials) != cudaSuccess || ptr == nullptr) {
        g_last_error = "pan2_mse_sums_noalloc: cudaGetSymbolAddress failed for the scratch array";
        return 3;
      }
      partials = static_cast<float*>(ptr);
      g_partials_addr[dev].store(partials, std::memory_order_release);
    }
  }
  // An error left by an earlier, unrelated launch is reported as such and left pending for its
  // owner (peek, not get), so it is never mistaken for a failure of this call.
  if (cudaPeekAtLastError() != cudaSuccess) {
    g_last_error = "pan2_mse_sums_noalloc: an earlier CUDA error is pending on this thread; nothing was launched";
    return 3;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int n_part = (int)(tiles > 0 ? tiles : 1);  // n == 0: one CTA writes a zero partial
  mse_tile_kernel<<<n_part, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(pred),
                                        static_cast<const __nv_bfloat16*>(target), n, partials);
  mse_final_kernel<<<1, 1024, 0, s>>>(partials, n_part, (float)n, out);
  if (cudaGetLastError() != cudaSuccess) {
    g_last_error = "pan2_mse_sums_noalloc: kernel launch failed";
    return 3;
  }
  return 0;
}

}  // extern "C"
