// Bandwidth-bound kernels of the decoder: RMSNorm, per-head q/k RMSNorm + RoPE, SwiGLU,
// embedding gather/scatter, and residual helpers.  All math in fp32, storage in bf16,
// 16-byte vector accesses where the row layout allows it.
#include "common.cuh"
#include "ops.h"

namespace trida {

// ------------------------------------------------------------------------------------------
// RMSNorm  y = x * rsqrt(mean(x^2) + eps) * w        (one warp per row)
// ------------------------------------------------------------------------------------------
__global__ void rmsnorm_fwd_kernel(const bf16* __restrict__ x, int64_t ldx, const bf16* __restrict__ w,
                                   bf16* __restrict__ y, int64_t ldy, float* __restrict__ rstd_out,
                                   int M, int D, float eps) {
  const int warps = blockDim.x >> 5;
  const int row = blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const bf16* xr = x + (int64_t)row * ldx;
  float ss = 0.f;
  for (int c = lane * 8; c < D; c += 256) {
    float f[8];
    load8(xr + c, f);
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += f[i] * f[i];
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / (float)D + eps);
  if (lane == 0 && rstd_out) rstd_out[row] = r;
  bf16* yr = y + (int64_t)row * ldy;
  for (int c = lane * 8; c < D; c += 256) {
    float f[8], g[8];
    load8(xr + c, f);
    load8(w + c, g);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = f[i] * r * g[i];
    store8(yr + c, f);
  }
}

// dx = r * (dy*w - xhat * mean(dy*w*xhat)) (+ dres);  dw += sum_rows dy*xhat   (fp32 atomics)
__global__ void rmsnorm_bwd_kernel(const bf16* __restrict__ dy, int64_t lddy, const bf16* __restrict__ x,
                                   int64_t ldx, const bf16* __restrict__ w, const float* __restrict__ rstd,
                                   const bf16* __restrict__ dres, int64_t lddres, bf16* __restrict__ dx,
                                   int64_t lddx, float* __restrict__ dw, int M, int D) {
  extern __shared__ float sdw_all[];  // [warps][D]: lane-owned columns, no atomics needed
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  float* sdw = sdw_all + (threadIdx.x >> 5) * D;
  for (int c = threadIdx.x; c < warps * D; c += blockDim.x) sdw_all[c] = 0.f;
  __syncthreads();
  for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < M; row += gridDim.x * warps) {
    const bf16* xr = x + (int64_t)row * ldx;
    const bf16* dyr = dy + (int64_t)row * lddy;
    const float r = rstd[row];
    float dot = 0.f;
    for (int c = lane * 8; c < D; c += 256) {
      float f[8], g[8], d[8];
      load8(xr + c, f);
      load8(w + c, g);
      load8(dyr + c, d);
#pragma unroll
      for (int i = 0; i < 8; ++i) dot += d[i] * g[i] * f[i] * r;
    }
    dot = warp_sum(dot) / (float)D;
    bf16* dxr = dx + (int64_t)row * lddx;
    for (int c = lane * 8; c < D; c += 256) {
      float f[8], g[8], d[8], o[8];
      load8(xr + c, f);
      load8(w + c, g);
      load8(dyr + c, d);
      if (dres) {
        load8(dres + (int64_t)row * lddres + c, o);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = 0.f;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float xh = f[i] * r;
        o[i] += r * (d[i] * g[i] - xh * dot);
        sdw[c + i] += d[i] * xh;
      }
      store8(dxr + c, o);
    }
  }
  __syncthreads();
  if (dw)
    for (int c = threadIdx.x; c < D; c += blockDim.x) {
      float t = 0.f;
      for (int wi = 0; wi < warps; ++wi) t += sdw_all[wi * D + c];
      atomicAdd(&dw[c], t);
    }
}

void rmsnorm_fwd(const bf16* x, int64_t ldx, const bf16* w, bf16* y, int64_t ldy, float* rstd, int M,
                 int D, float eps, cudaStream_t s) {
  const int warps = 8;
  rmsnorm_fwd_kernel<<<ceil_div(M, warps), warps * 32, 0, s>>>(x, ldx, w, y, ldy, rstd, M, D, eps);
}

void rmsnorm_bwd(const bf16* dy, int64_t lddy, const bf16* x, int64_t ldx, const bf16* w, const float* rstd,
                 const bf16* dres, int64_t lddres, bf16* dx, int64_t lddx, float* dw, int M, int D,
                 int sm_count, cudaStream_t s) {
  const int warps = 8;
  const size_t smem = (size_t)warps * D * sizeof(float);
  static size_t configured = 0;
  if (smem > 48 * 1024 && smem > configured) {
    cudaFuncSetAttribute(rmsnorm_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    configured = smem;
  }
  int blocks = ceil_div(M, warps * 4);
  blocks = blocks > sm_count * 2 ? sm_count * 2 : blocks;
  rmsnorm_bwd_kernel<<<blocks, warps * 32, smem, s>>>(dy, lddy, x, ldx, w, rstd, dres, lddres,
                                                                   dx, lddx, dw, M, D);
}

// ------------------------------------------------------------------------------------------
// Per-head RMSNorm of q and k followed by RoPE (half-split pairs (i, i+rd/2), rd <= d).
// qkv row layout: [Hq*d | Hkv*d | Hkv*d].  One warp per (token, head).  cos/sin tables are
// fp32 [max_pos, rd/2] indexed by the token's position.
// ------------------------------------------------------------------------------------------
__global__ void qk_norm_rope_fwd_kernel(const bf16* __restrict__ qkv, int64_t ldqkv,
                                        const bf16* __restrict__ qw, const bf16* __restrict__ kw,
                                        const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                                        const int* __restrict__ pos, bf16* __restrict__ q,
                                        bf16* __restrict__ k, float* __restrict__ rstd, int M, int Hq,
                                        int Hkv, int d, int rd, float eps, int qstride) {
  const int H = Hq + Hkv;
  const int64_t gw = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (gw >= (int64_t)M * H) return;
  const int tok = (int)(gw / H), h = (int)(gw % H);
  const bool is_q = h < Hq;
  const int64_t hcol = is_q ? (int64_t)h * qstride : (int64_t)Hq * qstride + (int64_t)(h - Hq) * d;
  const bf16* src = qkv + (int64_t)tok * ldqkv + hcol;
  const bf16* w = is_q ? qw : kw;
  bf16* dst = is_q ? (q + ((int64_t)tok * Hq + h) * d) : (k + ((int64_t)tok * Hkv + (h - Hq)) * d);
  // null norm weights: RoPE only (models without per-head q / k RMSNorm)
  float r = 1.f;
  if (w != nullptr) {
    float ss = 0.f;
    for (int c = lane; c < d; c += 32) {
      const float v = __bfloat162float(src[c]);
      ss += v * v;
    }
    ss = warp_sum(ss);
    r = rsqrtf(ss / (float)d + eps);
  }
  if (lane == 0) rstd[gw] = r;
  const int half = rd >> 1;
  const int p = pos[tok];
  const float* ct = cos_t + (int64_t)p * half;
  const float* st = sin_t + (int64_t)p * half;
  for (int i = lane; i < half; i += 32) {
    const float w1 = w != nullptr ? __bfloat162float(w[i]) : 1.f;
    const float w2 = w != nullptr ? __bfloat162float(w[i + half]) : 1.f;
    const float x1 = __bfloat162float(src[i]) * r * w1;
    const float x2 = __bfloat162float(src[i + half]) * r * w2;
    const float c = ct[i], s = st[i];
    dst[i] = __float2bfloat16(x1 * c - x2 * s);
    dst[i + half] = __float2bfloat16(x2 * c + x1 * s);
  }
  for (int i = rd + lane; i < d; i += 32)
    dst[i] = __float2bfloat16(__bfloat162float(src[i]) * r * (w != nullptr ? __bfloat162float(w[i]) : 1.f));
}

// Backward: dy (grad of the roped output) -> d(normalised) by the inverse rotation, then the
// RMSNorm backward.  Writes the q/k slices of dqkv; accumulates dqw/dkw (fp32 atomics).
__global__ void qk_norm_rope_bwd_kernel(const bf16* __restrict__ dq, const bf16* __restrict__ dk,
                                        const bf16* __restrict__ qkv, int64_t ldqkv,
                                        const bf16* __restrict__ qw, const bf16* __restrict__ kw,
                                        const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                                        const int* __restrict__ pos, const float* __restrict__ rstd,
                                        bf16* __restrict__ dqkv, int64_t lddqkv, float* __restrict__ dqw,
                                        float* __restrict__ dkw, int M, int Hq, int Hkv, int d, int rd,
                                        int qstride) {
  extern __shared__ float sdw_all[];  // [warps][2*d]: q weight grads then k weight grads
  const int nwarps = blockDim.x >> 5;
  float* sdw = sdw_all + (threadIdx.x >> 5) * 2 * d;
  for (int c = threadIdx.x; c < nwarps * 2 * d; c += blockDim.x) sdw_all[c] = 0.f;
  __syncthreads();
  const int H = Hq + Hkv;
  const int lane = threadIdx.x & 31;
  const int half = rd >> 1;
  const int64_t total = (int64_t)M * H;
  for (int64_t gw = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); gw < total;
       gw += (int64_t)gridDim.x * (blockDim.x >> 5)) {
    const int tok = (int)(gw / H), h = (int)(gw % H);
    const bool is_q = h < Hq;
    const int64_t hcol = is_q ? (int64_t)h * qstride : (int64_t)Hq * qstride + (int64_t)(h - Hq) * d;
    const bf16* src = qkv + (int64_t)tok * ldqkv + hcol;
    const bf16* w = is_q ? qw : kw;
    const bf16* g = is_q ? (dq + ((int64_t)tok * Hq + h) * d) : (dk + ((int64_t)tok * Hkv + (h - Hq)) * d);
    bf16* out = dqkv + (int64_t)tok * lddqkv + hcol;
    float* sw = sdw + (is_q ? 0 : d);
    const float r = rstd[gw];
    const int p = pos[tok];
    const float* ct = cos_t + (int64_t)p * half;
    const float* st = sin_t + (int64_t)p * half;
    // pass 1: dot = sum(dn * w * xhat) where dn = grad wrt the normalised (pre-rope) value
    float dot = 0.f;
    for (int i = lane; i < half; i += 32) {
      const float g1 = __bfloat162float(g[i]), g2 = __bfloat162float(g[i + half]);
      const float c = ct[i], s = st[i];
      const float dn1 = g1 * c + g2 * s, dn2 = g2 * c - g1 * s;
      dot += dn1 * __bfloat162float(w[i]) * __bfloat162float(src[i]) * r;
      dot += dn2 * __bfloat162float(w[i + half]) * __bfloat162float(src[i + half]) * r;
    }
    for (int i = rd + lane; i < d; i += 32)
      dot += __bfloat162float(g[i]) * __bfloat162float(w[i]) * __bfloat162float(src[i]) * r;
    dot = warp_sum(dot) / (float)d;
    for (int i = lane; i < half; i += 32) {
      const float g1 = __bfloat162float(g[i]), g2 = __bfloat162float(g[i + half]);
      const float c = ct[i], s = st[i];
      const float dn1 = g1 * c + g2 * s, dn2 = g2 * c - g1 * s;
      const float xh1 = __bfloat162float(src[i]) * r, xh2 = __bfloat162float(src[i + half]) * r;
      out[i] = __float2bfloat16(r * (dn1 * __bfloat162float(w[i]) - xh1 * dot));
      out[i + half] = __float2bfloat16(r * (dn2 * __bfloat162float(w[i + half]) - xh2 * dot));
      sw[i] += dn1 * xh1;
      sw[i + half] += dn2 * xh2;
    }
    for (int i = rd + lane; i < d; i += 32) {
      const float dn = __bfloat162float(g[i]);
      const float xh = __bfloat162float(src[i]) * r;
      out[i] = __float2bfloat16(r * (dn * __bfloat162float(w[i]) - xh * dot));
      sw[i] += dn * xh;
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < 2 * d; c += blockDim.x) {
    float t = 0.f;
    for (int wi = 0; wi < nwarps; ++wi) t += sdw_all[wi * 2 * d + c];
    float* dst = c < d ? (dqw ? dqw + c : nullptr) : (dkw ? dkw + (c - d) : nullptr);
    if (dst) atomicAdd(dst, t);
  }
}

void qk_norm_rope_fwd(const bf16* qkv, int64_t ldqkv, const bf16* qw, const bf16* kw, const float* cos_t,
                      const float* sin_t, const int* pos, bf16* q, bf16* k, float* rstd, int M, int Hq,
                      int Hkv, int d, int rd, float eps, int qstride, cudaStream_t s) {
  const int warps = 8;
  const int64_t total = (int64_t)M * (Hq + Hkv);
  qk_norm_rope_fwd_kernel<<<ceil_div(total, warps), warps * 32, 0, s>>>(qkv, ldqkv, qw, kw, cos_t, sin_t, pos,
                                                                       q, k, rstd, M, Hq, Hkv, d, rd, eps, qstride);
}

void qk_norm_rope_bwd(const bf16* dq, const bf16* dk, const bf16* qkv, int64_t ldqkv, const bf16* qw,
                      const bf16* kw, const float* cos_t, const float* sin_t, const int* pos,
                      const float* rstd, bf16* dqkv, int64_t lddqkv, float* dqw, float* dkw, int M, int Hq,
                      int Hkv, int d, int rd, int qstride, int sm_count, cudaStream_t s) {
  const int warps = 8;
  const int64_t total = (int64_t)M * (Hq + Hkv);
  int blocks = ceil_div(total, warps * 8);
  blocks = blocks > sm_count * 8 ? sm_count * 8 : blocks;
  qk_norm_rope_bwd_kernel<<<blocks, warps * 32, warps * 2 * d * sizeof(float), s>>>(
      dq, dk, qkv, ldqkv, qw, kw, cos_t, sin_t, pos, rstd, dqkv, lddqkv, dqw, dkw, M, Hq, Hkv, d, rd, qstride);
}

// ------------------------------------------------------------------------------------------
// Sigmoid output gate of the gated attention (Qwen3.5 full-attention layers):
//   y[t, h, :] = o[t, h, :] * sigmoid(gate[t, h, :]),  gate = qkv[t, h*2d + d : h*2d + 2d]
// ------------------------------------------------------------------------------------------
__global__ void attn_gate_fwd_kernel(const bf16* __restrict__ o, const bf16* __restrict__ qkv, int64_t ldqkv,
                                     bf16* __restrict__ y, int M, int Hq, int d) {
  const int vpr = Hq * d / 8;
  const int64_t total = (int64_t)M * vpr;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int row = (int)(i / vpr), c = (int)(i % vpr) * 8;
    const int h = c / d, e = c % d;
    float ov[8], gv[8], out[8];
    load8(o + (int64_t)row * Hq * d + c, ov);
    load8(qkv + (int64_t)row * ldqkv + (int64_t)h * 2 * d + d + e, gv);
#pragma unroll
    for (int j = 0; j < 8; ++j) out[j] = ov[j] / (1.f + __expf(-gv[j]));
    store8(y + (int64_t)row * Hq * d + c, out);
  }
}

__global__ void attn_gate_bwd_kernel(const bf16* __restrict__ dy, const bf16* __restrict__ o,
                                     const bf16* __restrict__ qkv, int64_t ldqkv, bf16* __restrict__ d_o,
                                     bf16* __restrict__ dqkv, int64_t lddqkv, int M, int Hq, int d) {
  const int vpr = Hq * d / 8;
  const int64_t total = (int64_t)M * vpr;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int row = (int)(i / vpr), c = (int)(i % vpr) * 8;
    const int h = c / d, e = c % d;
    float dv[8], ov[8], gv[8], dov[8], dgv[8];
    load8(dy + (int64_t)row * Hq * d + c, dv);
    load8(o + (int64_t)row * Hq * d + c, ov);
    load8(qkv + (int64_t)row * ldqkv + (int64_t)h * 2 * d + d + e, gv);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float sg = 1.f / (1.f + __expf(-gv[j]));
      dov[j] = dv[j] * sg;
      dgv[j] = dv[j] * ov[j] * sg * (1.f - sg);
    }
    store8(d_o + (int64_t)row * Hq * d + c, dov);
    store8(dqkv + (int64_t)row * lddqkv + (int64_t)h * 2 * d + d + e, dgv);
  }
}

void attn_gate_fwd(const bf16* o, const bf16* qkv, int64_t ldqkv, bf16* y, int M, int Hq, int d, int sm_count,
                   cudaStream_t s) {
  const int64_t total = (int64_t)M * Hq * d / 8;
  int blocks = ceil_div(total, 256);
  blocks = blocks > sm_count * 16 ? sm_count * 16 : blocks;
  attn_gate_fwd_kernel<<<blocks, 256, 0, s>>>(o, qkv, ldqkv, y, M, Hq, d);
}

void attn_gate_bwd(const bf16* dy, const bf16* o, const bf16* qkv, int64_t ldqkv, bf16* d_o, bf16* dqkv,
                   int64_t lddqkv, int M, int Hq, int d, int sm_count, cudaStream_t s) {
  const int64_t total = (int64_t)M * Hq * d / 8;
  int blocks = ceil_div(total, 256);
  blocks = blocks > sm_count * 16 ? sm_count * 16 : blocks;
  attn_gate_bwd_kernel<<<blocks, 256, 0, s>>>(dy, o, qkv, ldqkv, d_o, dqkv, lddqkv, M, Hq, d);
}

// ------------------------------------------------------------------------------------------
// SwiGLU on a [M, 2F] row = [gate | up]:  a = silu(g) * u
// ------------------------------------------------------------------------------------------
__global__ void swiglu_fwd_kernel(const bf16* __restrict__ gu, int64_t ldgu, bf16* __restrict__ a,
                                  int64_t lda, int M, int F) {
  const int vpr = F / 8;
  const int64_t total = (int64_t)M * vpr;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int row = (int)(i / vpr), c = (int)(i % vpr) * 8;
    float g[8], u[8], o[8];
    load8(gu + (int64_t)row * ldgu + c, g);
    load8(gu + (int64_t)row * ldgu + F + c, u);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = g[j] / (1.f + __expf(-g[j])) * u[j];
    store8(a + (int64_t)row * lda + c, o);
  }
}

__global__ void swiglu_bwd_kernel(const bf16* __restrict__ da, int64_t ldda, const bf16* __restrict__ gu,
                                  int64_t ldgu, bf16* __restrict__ dgu, int64_t lddgu, int M, int F) {
  const int vpr = F / 8;
  const int64_t total = (int64_t)M * vpr;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int row = (int)(i / vpr), c = (int)(i % vpr) * 8;
    float g[8], u[8], d[8], og[8], ou[8];
    load8(gu + (int64_t)row * ldgu + c, g);
    load8(gu + (int64_t)row * ldgu + F + c, u);
    load8(da + (int64_t)row * ldda + c, d);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float sg = 1.f / (1.f + __expf(-g[j]));
      const float silu = g[j] * sg;
      ou[j] = d[j] * silu;
      og[j] = d[j] * u[j] * sg * (1.f + g[j] * (1.f - sg));
    }
    store8(dgu + (int64_t)row * lddgu + c, og);
    store8(dgu + (int64_t)row * lddgu + F + c, ou);
  }
}

void swiglu_fwd(const bf16* gu, int64_t ldgu, bf16* a, int64_t lda, int M, int F, int sm_count, cudaStream_t s) {
  const int64_t total = (int64_t)M * (F / 8);
  int blocks = ceil_div(total, 256);
  blocks = blocks > sm_count * 16 ? sm_count * 16 : blocks;
  swiglu_fwd_kernel<<<blocks, 256, 0, s>>>(gu, ldgu, a, lda, M, F);
}

void swiglu_bwd(const bf16* da, int64_t ldda, const bf16* gu, int64_t ldgu, bf16* dgu, int64_t lddgu, int M,
                int F, int sm_count, cudaStream_t s) {
  const int64_t total = (int64_t)M * (F / 8);
  int blocks = ceil_div(total, 256);
  blocks = blocks > sm_count * 16 ? sm_count * 16 : blocks;
  swiglu_bwd_kernel<<<blocks, 256, 0, s>>>(da, ldda, gu, ldgu, dgu, lddgu, M, F);
}

// ------------------------------------------------------------------------------------------
// Embedding gather (forward) and fp32 scatter-add (backward).  One warp per token row.
// ------------------------------------------------------------------------------------------
__global__ void embed_fwd_kernel(const int64_t* __restrict__ ids, const bf16* __restrict__ table,
                                 bf16* __restrict__ out, int M, int D) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const bf16* src = table + ids[row] * (int64_t)D;
  bf16* dst = out + (int64_t)row * D;
  for (int c = lane * 8; c < D; c += 256)
    *reinterpret_cast<bf16x8*>(dst + c) = *reinterpret_cast<const bf16x8*>(src + c);
}

__global__ void embed_bwd_kernel(const int64_t* __restrict__ ids, const bf16* __restrict__ dout,
                                 float* __restrict__ dtable, int M, int D) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  float* dst = dtable + ids[row] * (int64_t)D;
  const bf16* src = dout + (int64_t)row * D;
  for (int c = lane * 8; c < D; c += 256) {
    float f[8];
    load8(src + c, f);
#pragma unroll
    for (int i = 0; i < 8; ++i) atomicAdd(dst + c + i, f[i]);
  }
}

void embed_fwd(const int64_t* ids, const bf16* table, bf16* out, int M, int D, cudaStream_t s) {
  embed_fwd_kernel<<<ceil_div(M, 8), 256, 0, s>>>(ids, table, out, M, D);
}

void embed_bwd(const int64_t* ids, const bf16* dout, float* dtable, int M, int D, cudaStream_t s) {
  embed_bwd_kernel<<<ceil_div(M, 8), 256, 0, s>>>(ids, dout, dtable, M, D);
}

}  // namespace trida
