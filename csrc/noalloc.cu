// Allocation-free variant of the global gradient-norm entry point (see trida_noalloc.h).
// Its scratch is a file-scope __device__ array; host code obtains that array's device address per
// device with cudaGetSymbolAddress (the host-side name is only a stand-in, never a device address).
#include <cstdint>
#include <mutex>

#include "ops.h"
#include "trida_noalloc.h"

namespace {

constexpr int kBlocksPerBuffer = 256;   // partial sums per gradient buffer (as the regular entry point)
constexpr int kMaxDevices = 64;

static __device__ __align__(256) float g_partial_scratch[TRIDA_NOALLOC_MAX_BUFFERS * kBlocksPerBuffer];

std::mutex g_mu;
float* g_scratch_ptr[kMaxDevices] = {nullptr};

// Device address of the scratch array on the current device, looked up once per device.
int scratch_for_current_device(float** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return TRIDA_NOALLOC_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_partial_scratch) != cudaSuccess || p == nullptr)
      return TRIDA_NOALLOC_ERR_SYMBOL_ADDRESS;
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_ptr[dev];
  return TRIDA_NOALLOC_OK;
}

}  // namespace

extern "C" int trida_grad_norm_noalloc(const float* const* grads, const long long* numels, int n_buffers,
                                       float max_norm, float* norm_out, float* coef_out, cudaStream_t stream) {
  if (grads == nullptr || numels == nullptr || norm_out == nullptr || coef_out == nullptr || n_buffers <= 0)
    return TRIDA_NOALLOC_ERR_INVALID_ARGUMENT;
  if (n_buffers > TRIDA_NOALLOC_MAX_BUFFERS) return TRIDA_NOALLOC_ERR_TOO_MANY_BUFFERS;
  // The partial-sum kernel reads whole float4 vectors, so every buffer must start on a 16-byte
  // boundary; an offset view would fault the caller's context.  Rejected before anything launches.
  for (int i = 0; i < n_buffers; ++i)
    if (grads[i] == nullptr || numels[i] < 0 || (reinterpret_cast<uintptr_t>(grads[i]) & 15u) != 0)
      return TRIDA_NOALLOC_ERR_INVALID_ARGUMENT;
  // An error left pending by the caller's own work would otherwise be reported (and cleared) as
  // this call's launch failure.
  if (cudaPeekAtLastError() != cudaSuccess) return TRIDA_NOALLOC_ERR_PENDING;
  float* scratch = nullptr;
  const int rc = scratch_for_current_device(&scratch);
  if (rc != TRIDA_NOALLOC_OK) return rc;
  for (int i = 0; i < n_buffers; ++i)
    trida::sumsq_partial(grads[i], (int64_t)numels[i], scratch + (size_t)i * kBlocksPerBuffer, kBlocksPerBuffer,
                         stream);
  trida::clip_coef(scratch, n_buffers * kBlocksPerBuffer, max_norm, norm_out, coef_out, stream);
  return cudaGetLastError() == cudaSuccess ? TRIDA_NOALLOC_OK : TRIDA_NOALLOC_ERR_LAUNCH;
}

extern "C" const char* trida_noalloc_error_string(int code) {
  switch (code) {
    case TRIDA_NOALLOC_OK: return "ok";
    case TRIDA_NOALLOC_ERR_INVALID_ARGUMENT:
      return "invalid argument (null or not 16-byte aligned gradient pointer, negative size or n_buffers <= 0)";
    case TRIDA_NOALLOC_ERR_TOO_MANY_BUFFERS:
      return "too many gradient buffers: at most TRIDA_NOALLOC_MAX_BUFFERS (64) per call";
    case TRIDA_NOALLOC_ERR_NO_DEVICE: return "no current CUDA device";
    case TRIDA_NOALLOC_ERR_SYMBOL_ADDRESS: return "cudaGetSymbolAddress failed for the scratch array";
    case TRIDA_NOALLOC_ERR_LAUNCH: return "kernel launch failed";
    case TRIDA_NOALLOC_ERR_PENDING:
      return "a CUDA error from earlier work was already pending on entry (left in place; nothing launched)";
    default: return "unknown error code";
  }
}
