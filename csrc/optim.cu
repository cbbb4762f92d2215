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

// Eight elements per thread and step: one 16-byte load of bf16 parameters and two of each fp32
// stream (gradient, m, v), all issued before the math, so a thread keeps 112 bytes in flight.
// The fp32 streams are touched once per step and use evict-first cache hints.
__device__ __forceinline__ float4 ld_cs4(const float* p) { return __ldcs(reinterpret_cast<const float4*>(p)); }
__device__ __forceinline__ void st_cs4(float* p, float4 v) { __stcs(reinterpret_cast<float4*>(p), v); }

__global__ void __launch_bounds__(256) adamw_bf16_vec_kernel(bf16* __restrict__ param, const float* __restrict__ grad,
                                                             float* __restrict__ m, float* __restrict__ v, int64_t n8,
                                                             float lr, float b1, float b2, float eps, float wd,
                                                             float bc1, float bc2_sqrt, const float* __restrict__ coef) {
  const float c = coef ? *coef : 1.f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = i * 8;
    const uint4 praw = *reinterpret_cast<const uint4*>(param + e);
    const float4 g0 = ld_cs4(grad + e), g1 = ld_cs4(grad + e + 4);
    const float4 m0 = ld_cs4(m + e), m1 = ld_cs4(m + e + 4);
    const float4 v0 = ld_cs4(v + e), v1 = ld_cs4(v + e + 4);
    float pf[8], gf[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
    float mf[8] = {m0.x, m0.y, m0.z, m0.w, m1.x, m1.y, m1.z, m1.w};
    float vf[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    const __nv_bfloat162* p2 = reinterpret_cast<const __nv_bfloat162*>(&praw);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 t = __bfloat1622float2(p2[k]);
      pf[2 * k] = t.x;
      pf[2 * k + 1] = t.y;
    }
    uint4 pout;
    __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&pout);
#pragma unroll
    for (int k = 0; k < 8; ++k) pf[k] = adamw_one(pf[k], gf[k] * c, mf[k], vf[k], lr, b1, b2, eps, wd, bc1, bc2_sqrt);
#pragma unroll
    for (int k = 0; k < 4; ++k) o2[k] = __floats2bfloat162_rn(pf[2 * k], pf[2 * k + 1]);
    *reinterpret_cast<uint4*>(param + e) = pout;
    st_cs4(m + e, make_float4(mf[0], mf[1], mf[2], mf[3]));
    st_cs4(m + e + 4, make_float4(mf[4], mf[5], mf[6], mf[7]));
    st_cs4(v + e, make_float4(vf[0], vf[1], vf[2], vf[3]));
    st_cs4(v + e + 4, make_float4(vf[4], vf[5], vf[6], vf[7]));
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
  const bool vec = ((reinterpret_cast<uintptr_t>(param) | reinterpret_cast<uintptr_t>(grad) |
                    reinterpret_cast<uintptr_t>(m) | reinterpret_cast<uintptr_t>(v)) & 15) == 0;
  const int64_t n8 = vec ? n / 8 : 0;
  if (n8 > 0) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    int64_t blocks = (n8 + 255) / 256;
    blocks = blocks > (int64_t)sms * 8 ? (int64_t)sms * 8 : blocks;
    adamw_bf16_vec_kernel<<<(int)blocks, 256, 0, s>>>(param, grad, m, v, n8, lr, beta1, beta2, eps, wd, bc1,
                                                      sqrtf(bc2), coef);
  }
  const int64_t done = n8 * 8;
  if (done < n)   // tail (or unaligned buffers): one element per thread
    adamw_bf16_kernel<<<adam_blocks(n - done), 256, 0, s>>>(param + done, grad + done, m + done, v + done, n - done,
                                                            lr, beta1, beta2, eps, wd, bc1, sqrtf(bc2), coef);
}

}  // namespace trida
