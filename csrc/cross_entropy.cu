// Row kernel of the fused linear cross-entropy: given one chunk of fp32 logits (produced by the
// tensor-core GEMM h . W^T), compute per-row CE = logsumexp(z) - z[target] and, in the same pass
// over the row, the logit gradient (softmax(z) - onehot) * weight * grad_scale in bf16, which feeds
// the dH and dW GEMMs.  The full [N, V] logit matrix never exists: the caller walks row chunks.
#include "common.cuh"
#include "ops.h"

namespace trida {

__global__ void __launch_bounds__(512) ce_rows_kernel(const float* __restrict__ logits, int64_t ld,
                                                      const int64_t* __restrict__ target,
                                                      const float* __restrict__ weight, float grad_scale, int V,
                                                      float* __restrict__ loss, bf16* __restrict__ dlogits,
                                                      int64_t ldd) {
  __shared__ float red[32];
  const int row = blockIdx.x;
  const float* z = logits + (int64_t)row * ld;
  // pass 1: per-thread online (max, sum) over float4 vectors
  float m = -INFINITY, s = 0.f;
  const int nv = V / 4;
  for (int i = threadIdx.x; i < nv; i += blockDim.x) {
    const float4 v = reinterpret_cast<const float4*>(z)[i];
    const float mx = fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w));
    if (mx > m) {
      s *= __expf(m - mx);
      m = mx;
    }
    s += __expf(v.x - m) + __expf(v.y - m) + __expf(v.z - m) + __expf(v.w - m);
  }
  for (int i = nv * 4 + threadIdx.x; i < V; i += blockDim.x) {
    const float x = z[i];
    if (x > m) {
      s *= __expf(m - x);
      m = x;
    }
    s += __expf(x - m);
  }
  const float gm = block_max(m, red);
  s = (m == -INFINITY) ? 0.f : s * __expf(m - gm);
  const float gs = block_sum(s, red);
  const float lse = gm + logf(gs);
  const int64_t tgt = target[row];
  if (threadIdx.x == 0) loss[row] = lse - z[tgt];
  if (dlogits == nullptr) return;
  const float w = (weight ? weight[row] : 1.f) * grad_scale;
  bf16* dz = dlogits + (int64_t)row * ldd;
  for (int i = threadIdx.x; i < nv; i += blockDim.x) {
    const float4 v = reinterpret_cast<const float4*>(z)[i];
    const int c = i * 4;
    float g0 = __expf(v.x - lse), g1 = __expf(v.y - lse), g2 = __expf(v.z - lse), g3 = __expf(v.w - lse);
    if (tgt >= c && tgt < c + 4) {
      const int o = (int)(tgt - c);
      if (o == 0) g0 -= 1.f; else if (o == 1) g1 -= 1.f; else if (o == 2) g2 -= 1.f; else g3 -= 1.f;
    }
    __nv_bfloat162 a = __floats2bfloat162_rn(g0 * w, g1 * w), b = __floats2bfloat162_rn(g2 * w, g3 * w);
    uint2 pk;
    pk.x = *reinterpret_cast<uint32_t*>(&a);
    pk.y = *reinterpret_cast<uint32_t*>(&b);
    *reinterpret_cast<uint2*>(dz + c) = pk;
  }
  for (int i = nv * 4 + threadIdx.x; i < V; i += blockDim.x) {
    float g = __expf(z[i] - lse);
    if (i == tgt) g -= 1.f;
    dz[i] = __float2bfloat16(g * w);
  }
}

void ce_rows_fwd_bwd(const float* logits, int64_t ld, const int64_t* target, const float* weight, float grad_scale,
                     int n, int V, float* loss, bf16* dlogits, int64_t ldd, cudaStream_t s) {
  if (n <= 0) return;
  ce_rows_kernel<<<n, 512, 0, s>>>(logits, ld, target, weight, grad_scale, V, loss, dlogits, ldd);
}

}  // namespace trida
