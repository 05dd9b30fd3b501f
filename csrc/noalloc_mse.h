// C interface of the allocation-free loss-sum entry point (implemented in noalloc_mse.cu).
//
// This entry point has no counterpart in the reference project.  It is for callers that cannot
// call cudaMalloc or any routine that allocates device memory behind their back: runtimes and
// custom allocators that own every device allocation and forbid hidden ones, and C/C++ programs
// that link this library without PyTorch and so have no caching allocator to borrow scratch
// space from.  The caller passes device pointers for every input and output; the only scratch is
// a fixed 64 KB array inside the library.
#pragma once

#ifdef __cplusplus
extern "C" {
#endif

// out[0] = sum over i < n of (pred[i] - target[i])^2 and out[1] = n, in fp32, on `stream`
// (a cudaStream_t, or null for the default stream).  `pred` and `target` are bf16 device
// arrays of n elements, 16-byte aligned, n a multiple of 8 and at most 33,554,432; `out` is a
// device array of two floats.
//
// Returns 0 on success, 1 for bad arguments, 2 when n exceeds the scratch limit, 3 on a CUDA
// error; pan2_noalloc_last_error() then describes the failure.
//
// The first call on each device looks up the scratch array's device address with that device
// current; make that first call before any stream capture begins.  All calls share the scratch
// array, so calls whose kernels overlap on the GPU (for example on two streams at once) race and
// must be ordered by the caller.
int pan2_mse_sums_noalloc(const void* pred, const void* target, long long n, float* out, void* stream);

// Message of the last failed pan2_mse_sums_noalloc call on the calling host thread.
const char* pan2_noalloc_last_error(void);

#ifdef __cplusplus
}
#endif
