// Optimizer kernels over flat parameter buffers: global gradient norm (two-stage, deterministic),
// clip coefficient computed on the device (no host sync), and fused AdamW that applies the clip
// coefficient, updates fp32 moments and the master weights, and writes the bf16 compute copy.
#include "common.cuh"
#include "ops.h"

namespace trida {

__global__ void sumsq_kernel(const float* __restrict__ g, int64_t n, float* __restrict__ partial) {
  __shared__ float red[32];
  float acc = 0.f;
  const int64_t n4 = n / 4;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    const float4 v = reinterpret_cast<const float4*>(g)[i];
    acc += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  for (int64_t i = n4 * 4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    acc += g[i] * g[i];
  acc = block_sum(acc, red);
  if (threadIdx.x == 0) partial[blockIdx.x] = acc;
}

// partial may hold several buffers' partials back to back (nblocks total).
__global__ void clip_coef_kernel(const float* __restrict__ partial, int nblocks, float max_norm,
                                 float* __restrict__ norm_out, float* __restrict__ coef_out) {
  __shared__ float red[32];
  float acc = 0.f;
  for (int i = threadIdx.x; i < nblocks; i += blockDim.x) acc += partial[i];
  acc = block_sum(acc, red);
  if (threadIdx.x == 0) {
    const float norm = sqrtf(acc);
    *norm_out = norm;
    // torch.nn.utils.clip_grad_norm_: coef = max_norm / (norm + 1e-6), clamped to 1
    const float c = max_norm / (norm + 1e-6f);
    *coef_out = c < 1.f ? c : 1.f;
  }
}

void sumsq_partial(const float* g, int64_t n, float* partial, int nblocks, cudaStream_t s) {
  sumsq_kernel<<<nblocks, 512, 0, s>>>(g, n, partial);
}

void clip_coef(const float* partial, int nblocks, float max_norm, float* norm_out, float* coef_out, cudaStream_t s) {
  clip_coef_kernel<<<1, 1024, 0, s>>>(partial, nblocks, max_norm, norm_out, coef_out);
}

// torch.optim.AdamW (decoupled weight decay, bias-corrected moments).
__device__ __forceinline__ float adamw_one(float p, float g, float& m, float& v, float lr, float b1, float b2,
                                           float eps, float wd, float bc1, float bc2_sqrt) {
  p *= (1.f - lr * wd);
  m = b1 * m + (1.f - b1) * g;
  v = b2 * v + (1.f - b2) * g * g;
  const float denom = sqrtf(v) / bc2_sqrt + eps;
  return p - (lr / bc1) * (m / denom);
}

__global__ void adamw_master_kernel(float* __restrict__ master, bf16* __restrict__ pbf, const float* __restrict__ grad,
                                    float* __restrict__ m, float* __restrict__ v, int64_t n, float lr, float b1,
                                    float b2, float eps, float wd, float bc1, float bc2_sqrt,
                                    const float* __restrict__ coef) {
  const float c = coef ? *coef : 1.f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float mi = m[i], vi = v[i];
    const float p = adamw_one(master[i], grad[i] * c, mi, vi, lr, b1, b2, eps, wd, bc1, bc2_sqrt);
    m[i] = mi;
    v[i] = vi;
    master[i] = p;
    if (pbf) pbf[i] = __float2bfloat16(p);
  }
}

__global__ void adamw_bf16_kernel(bf16* __restrict__ param, const float* __restrict__ grad, float* __restrict__ m,
                                  float* __restrict__ v, int64_t n, float lr, float b1, float b2, float eps, float wd,
                                  float bc1, float bc2_sqrt, const float* __restrict__ coef) {
  const float c = coef ? *coef : 1.f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float mi = m[i], vi = v[i];
    const float p = adamw_one(__bfloat162float(param[i]), grad[i] * c, mi, vi, lr, b1, b2, eps, wd, bc1, bc2_sqrt);
    m[i] = mi;
    v[i] = vi;
    param[i] = __float2bfloat16(p);
  }
}

static int adam_blocks(int64_t n) {
  int64_t b = (n + 255) / 256;
  return (int)(b > 148 * 32 ? 148 * 32 : (b < 1 ? 1 : b));
}

void adamw_step(float* master, bf16* param_bf16, const float* grad, float* m, float* v, int64_t n, float lr,
                float beta1, float beta2, float eps, float wd, int step, const float* coef, cudaStream_t s) {
  const float bc1 = 1.f - powf(beta1, (float)step), bc2 = 1.f - powf(beta2, (float)step);
  adamw_master_kernel<<<adam_blocks(n), 256, 0, s>>>(master, param_bf16, grad, m, v, n, lr, beta1, beta2, eps, wd,
                                                     bc1, sqrtf(bc2), coef);
}

void adamw_step_bf16(bf16* param, const float* grad, float* m, float* v, int64_t n, float lr, float beta1,
                     float beta2, float eps, float wd, int step, const float* coef, cudaStream_t s) {
  const float bc1 = 1.f - powf(beta1, (float)step), bc2 = 1.f - powf(beta2, (float)step);
  adamw_bf16_kernel<<<adam_blocks(n), 256, 0, s>>>(param, grad, m, v, n, lr, beta1, beta2, eps, wd, bc1, sqrtf(bc2),
                                                   coef);
}

}  // namespace trida
