/*
 * Allocation-free C entry point of the global gradient-norm / clip-coefficient kernels.
 *
 * This interface has no counterpart in the reference (trida-stack has no native code at all).
 * It exists for callers that cannot allocate device memory: runtimes or custom allocators that
 * own all device memory and forbid cudaMalloc/cudaFree on their hot path, and non-PyTorch hosts
 * (plain C/C++ training loops) that link this library without the PyTorch caching allocator and
 * have no allocator of their own to hand it.  The regular entry point gets its
 * partial-sum scratch from PyTorch; this one uses a fixed scratch array compiled into the library
 * instead, so it calls no cudaMalloc, cudaFree or any allocating library routine.
 *
 * Limits and behaviour:
 *   - At most TRIDA_NOALLOC_MAX_BUFFERS gradient buffers per call (larger counts are rejected
 *     with TRIDA_NOALLOC_ERR_TOO_MANY_BUFFERS and nothing is launched).
 *   - The scratch array (TRIDA_NOALLOC_MAX_BUFFERS * 256 floats = 64 KiB) lives in every GPU that
 *     loads the library until the process exits.
 *   - The first call on a device looks up the scratch array's device address for that device
 *     (cudaGetSymbolAddress, with that device current).  Make that first call before any stream
 *     capture begins.
 *   - All calls share the one scratch array: two calls whose kernels overlap on the GPU (for
 *     example on different streams without ordering between them) race and give wrong results.
 *     Each call overwrites every scratch value it reads, so nothing needs clearing between calls.
 *   - The caller passes and owns every input (device pointers to fp32 gradient buffers, their
 *     element counts on the host) and both outputs (one device float each).
 *   - Every gradient pointer must be 16-byte aligned (the kernels read float4 vectors).  A null or
 *     misaligned pointer, a negative size or n_buffers <= 0 returns
 *     TRIDA_NOALLOC_ERR_INVALID_ARGUMENT before anything is launched.
 *   - A CUDA error already pending on entry (from the caller's own earlier work) is left in place
 *     and reported as TRIDA_NOALLOC_ERR_PENDING; nothing is launched.
 *   - The scratch address is looked up once per device number and cached for the life of the
 *     process, so only each device's primary context is supported (the CUDA runtime's default,
 *     also PyTorch's), and the device must not be reset (cudaDeviceReset) after the first call.
 */
#ifndef TRIDA_NOALLOC_H_
#define TRIDA_NOALLOC_H_

#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TRIDA_NOALLOC_MAX_BUFFERS 64

#define TRIDA_NOALLOC_OK 0
#define TRIDA_NOALLOC_ERR_INVALID_ARGUMENT 1
#define TRIDA_NOALLOC_ERR_TOO_MANY_BUFFERS 2
#define TRIDA_NOALLOC_ERR_NO_DEVICE 3
#define TRIDA_NOALLOC_ERR_SYMBOL_ADDRESS 4
#define TRIDA_NOALLOC_ERR_LAUNCH 5
#define TRIDA_NOALLOC_ERR_PENDING 6

/* norm_out = ||concat(grads)||_2 ; coef_out = min(1, max_norm / (norm + 1e-6)), both written on
 * the device in stream order (no host synchronisation).  Returns TRIDA_NOALLOC_OK or an error. */
int trida_grad_norm_noalloc(const float* const* grads, const long long* numels, int n_buffers, float max_norm,
                            float* norm_out, float* coef_out, cudaStream_t stream);

/* Human-readable text for a return code of trida_grad_norm_noalloc. */
const char* trida_noalloc_error_string(int code);

#ifdef __cplusplus
}
#endif

#endif /* TRIDA_NOALLOC_H_ */
