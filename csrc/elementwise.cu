// Bandwidth-bound kernels of the decoder: RMSNorm, per-head q/k RMSNorm + RoPE, SwiGLU,
// embedding gather/scatter, and residual helpers.  All math in fp32, storage in bf16,
// 16-byte vector accesses where the row layout allows it.
#include <initializer_list>

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

// Row-per-CTA variants for D = 256 k (<= 8192 forward, <= 5120 backward): D / 8 threads (forward:
// D / 16 when D is a multiple of 512, two vectors each), each owning the same columns of every row it
// visits (16-byte accesses), grid-stride over rows with the next row's loads issued before the
// current row's block reduction, so every thread keeps two
// rows of loads in flight.  The per-row sum goes through a double-buffered shared slot per warp
// (one barrier per row).  The backward keeps its columns of dw in registers across all rows
// and adds them once per CTA.
__device__ __forceinline__ bf16x8 ld_stream8(const bf16* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return *reinterpret_cast<bf16x8*>(&v);
}

__device__ __forceinline__ void unpack8(const bf16x8& v, float (&f)[8]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(v.h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

// sum of v over the CTA; red holds 2 x 32 floats, par alternates per call
__device__ __forceinline__ float cta_row_sum(float v, float (*red)[32], int par) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) red[par][threadIdx.x >> 5] = v;
  __syncthreads();
  const int nw = blockDim.x >> 5;
  float t = 0.f;
  for (int i = 0; i < nw; ++i) t += red[par][i];
  return t;
}

template <int VPT>
__global__ void __launch_bounds__(1024) rmsnorm_fwd_cta_kernel(const bf16* __restrict__ x, int64_t ldx,
                                                               const bf16* __restrict__ w, bf16* __restrict__ y,
                                                               int64_t ldy, float* __restrict__ rstd_out, int M,
                                                               float eps) {
  // VPT 16-byte vectors per thread, vector v at element (v * blockDim.x + threadIdx.x) * 8
  __shared__ float red[2][32];
  const int D = blockDim.x * 8 * VPT;
  int e[VPT];
  float g[VPT][8];
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    e[v] = (v * blockDim.x + threadIdx.x) * 8;
    load8(w + e[v], g[v]);
  }
  int row = blockIdx.x, par = 0;
  bf16x8 cur[VPT];
#pragma unroll
  for (int v = 0; v < VPT; ++v) cur[v] = row < M ? ld_stream8(x + (int64_t)row * ldx + e[v]) : bf16x8{};
  for (; row < M; row += gridDim.x, par ^= 1) {
    const int nrow = row + gridDim.x;
    bf16x8 nxt[VPT];
#pragma unroll
    for (int v = 0; v < VPT; ++v) nxt[v] = nrow < M ? ld_stream8(x + (int64_t)nrow * ldx + e[v]) : bf16x8{};
    float f[VPT][8];
    float ss = 0.f;
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
      unpack8(cur[v], f[v]);
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += f[v][i] * f[v][i];
    }
    const float r = rsqrtf(cta_row_sum(ss, red, par) / (float)D + eps);
    if (threadIdx.x == 0 && rstd_out) rstd_out[row] = r;
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
#pragma unroll
      for (int i = 0; i < 8; ++i) f[v][i] = f[v][i] * r * g[v][i];
      store8(y + (int64_t)row * ldy + e[v], f[v]);
      cur[v] = nxt[v];
    }
  }
}

template <int VPT>
__global__ void __launch_bounds__(VPT == 2 ? 320 : 640) rmsnorm_bwd_cta_kernel(const bf16* dy, int64_t lddy, const bf16* x,
                                                               int64_t ldx, const bf16* __restrict__ w,
                                                               const float* __restrict__ rstd, const bf16* dres,
                                                               int64_t lddres, bf16* dx, int64_t lddx,
                                                               float* __restrict__ dw, int M) {
  __shared__ float red[2][32];
  const int D = blockDim.x * 8 * VPT;
  int e[VPT];
  float g[VPT][8], acc[VPT][8];
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    e[v] = (v * blockDim.x + threadIdx.x) * 8;
    load8(w + e[v], g[v]);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[v][i] = 0.f;
  }
  int row = blockIdx.x, par = 0;
  bf16x8 cx[VPT], cd[VPT], cr[VPT];
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    cx[v] = bf16x8{}; cd[v] = bf16x8{}; cr[v] = bf16x8{};
    if (row < M) {
      cx[v] = ld_stream8(x + (int64_t)row * ldx + e[v]);
      cd[v] = ld_stream8(dy + (int64_t)row * lddy + e[v]);
      if (dres) cr[v] = ld_stream8(dres + (int64_t)row * lddres + e[v]);
    }
  }
  for (; row < M; row += gridDim.x, par ^= 1) {
    const int nrow = row + gridDim.x;
    bf16x8 nx[VPT], nd[VPT], nr[VPT];
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
      nx[v] = bf16x8{}; nd[v] = bf16x8{}; nr[v] = bf16x8{};
      if (nrow < M) {
        nx[v] = ld_stream8(x + (int64_t)nrow * ldx + e[v]);
        nd[v] = ld_stream8(dy + (int64_t)nrow * lddy + e[v]);
        if (dres) nr[v] = ld_stream8(dres + (int64_t)nrow * lddres + e[v]);
      }
    }
    const float r = rstd[row];
    float f[VPT][8], d[VPT][8];
    float dot = 0.f;
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
      unpack8(cx[v], f[v]);
      unpack8(cd[v], d[v]);
#pragma unroll
      for (int i = 0; i < 8; ++i) dot += d[v][i] * g[v][i] * f[v][i];
    }
    dot = cta_row_sum(dot, red, par) * r / (float)D;
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
      float o[8];
      if (dres) {
        unpack8(cr[v], o);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = 0.f;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float xh = f[v][i] * r;
        o[i] += r * (d[v][i] * g[v][i] - xh * dot);
        acc[v][i] += d[v][i] * xh;
      }
      store8(dx + (int64_t)row * lddx + e[v], o);
      cx[v] = nx[v];
      cd[v] = nd[v];
      cr[v] = nr[v];
    }
  }
  if (dw && blockIdx.x < M) {
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
      atomicAdd(reinterpret_cast<float4*>(dw + e[v]), make_float4(acc[v][0], acc[v][1], acc[v][2], acc[v][3]));
      atomicAdd(reinterpret_cast<float4*>(dw + e[v] + 4), make_float4(acc[v][4], acc[v][5], acc[v][6], acc[v][7]));
    }
  }
}

static int cta_row_blocks(const void* kernel, int threads, int M) {
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  }
  int per_sm = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, 0);
  const int blocks = sms * (per_sm > 0 ? per_sm : 1);
  return blocks < M ? blocks : (M > 0 ? M : 1);
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

static bool cta_row_ok(int D, int max_threads) { return D % 256 == 0 && D / 8 <= max_threads; }

void rmsnorm_fwd(const bf16* x, int64_t ldx, const bf16* w, bf16* y, int64_t ldy, float* rstd, int M,
                 int D, float eps, cudaStream_t s) {
  const int warps = 8;
  if (cta_row_ok(D, 1024) && ldx % 8 == 0 && ldy % 8 == 0 && aligned16(x) && aligned16(y) && aligned16(w)) {
    if (D % 512 == 0) {   // two vectors per thread: half the per-row reduction work per byte
      const int threads = D / 16;
      rmsnorm_fwd_cta_kernel<2><<<cta_row_blocks((const void*)rmsnorm_fwd_cta_kernel<2>, threads, M), threads, 0,
                                  s>>>(x, ldx, w, y, ldy, rstd, M, eps);
    } else {
      const int threads = D / 8;
      rmsnorm_fwd_cta_kernel<1><<<cta_row_blocks((const void*)rmsnorm_fwd_cta_kernel<1>, threads, M), threads, 0,
                                  s>>>(x, ldx, w, y, ldy, rstd, M, eps);
    }
    return;
  }
  rmsnorm_fwd_kernel<<<ceil_div(M, warps), warps * 32, 0, s>>>(x, ldx, w, y, ldy, rstd, M, D, eps);
}

void rmsnorm_bwd(const bf16* dy, int64_t lddy, const bf16* x, int64_t ldx, const bf16* w, const float* rstd,
                 const bf16* dres, int64_t lddres, bf16* dx, int64_t lddx, float* dw, int M, int D,
                 int sm_count, cudaStream_t s) {
  const int warps = 8;
  if (cta_row_ok(D, 640) && lddy % 8 == 0 && ldx % 8 == 0 && lddx % 8 == 0 && (!dres || lddres % 8 == 0) &&
      aligned16(dy) && aligned16(x) && aligned16(w) && aligned16(dx) && (!dres || aligned16(dres)) &&
      (!dw || aligned16(dw))) {
    // one vector per thread: two (137 registers, 0.67 of HBM) lose to one (91 registers, 0.77)
    const int threads = D / 8;
    rmsnorm_bwd_cta_kernel<1><<<cta_row_blocks((const void*)rmsnorm_bwd_cta_kernel<1>, threads, M), threads, 0,
                                s>>>(dy, lddy, x, ldx, w, rstd, dres, lddres, dx, lddx, dw, M);
    return;
  }
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

// Vector variants for d in {64, 128, 256} and rd a multiple of 16: one warp per token walks all
// its heads, d / 8 lanes to a head (8 consecutive elements and one 16-byte access per lane), so
// 32 / (d / 8) heads move per step and four steps' loads are issued together.  The token's
// position, its cos / sin values and both norm weights are read once per token.  The RoPE
// partner of element e < rd/2 is e + rd/2, rd/16 lanes away in the same head, fetched with one
// shuffle; per-head sums reduce over the head's d / 8 lanes.
template <int D>
struct QkLane {
  static constexpr int LPH = D / 8, HPW = 32 / LPH;
  int sub, e0, partner;
  bool roped, first;
  __device__ QkLane(int lane, int rd) {
    sub = lane / LPH;
    const int j = lane % LPH, hl = rd >> 4;
    e0 = j * 8;
    roped = e0 < rd;
    first = e0 < (rd >> 1);
    partner = sub * LPH + (roped ? (first ? j + hl : j - hl) : j);
  }
};

__device__ __forceinline__ void load_rope8(const float* cos_t, const float* sin_t, int64_t base, float (&c)[8],
                                           float (&sn)[8]) {
  const float4 c0 = *reinterpret_cast<const float4*>(cos_t + base);
  const float4 c1 = *reinterpret_cast<const float4*>(cos_t + base + 4);
  const float4 s0 = *reinterpret_cast<const float4*>(sin_t + base);
  const float4 s1 = *reinterpret_cast<const float4*>(sin_t + base + 4);
  c[0] = c0.x; c[1] = c0.y; c[2] = c0.z; c[3] = c0.w; c[4] = c1.x; c[5] = c1.y; c[6] = c1.z; c[7] = c1.w;
  sn[0] = s0.x; sn[1] = s0.y; sn[2] = s0.z; sn[3] = s0.w; sn[4] = s1.x; sn[5] = s1.y; sn[6] = s1.z; sn[7] = s1.w;
}

template <int D>
__global__ void __launch_bounds__(256, 3) qk_norm_rope_fwd_vec_kernel(
    const bf16* __restrict__ qkv, int64_t ldqkv, const bf16* __restrict__ qw, const bf16* __restrict__ kw,
    const float* __restrict__ cos_t, const float* __restrict__ sin_t, const int* __restrict__ pos,
    bf16* __restrict__ q, bf16* __restrict__ k, float* __restrict__ rstd, int M, int Hq, int Hkv, int rd,
    float eps, int qstride) {
  using L = QkLane<D>;
  constexpr int UNR = 4;
  const int tok = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (tok >= M) return;  // warp-uniform
  const L ln(threadIdx.x & 31, rd);
  const int H = Hq + Hkv, half = rd >> 1;
  const bool norm = qw != nullptr;
  float c[8], sn[8];
  if (ln.roped) load_rope8(cos_t, sin_t, (int64_t)pos[tok] * half + (ln.first ? ln.e0 : ln.e0 - half), c, sn);
  // the norm weights stay packed (bf16 pairs) and the loads in flight stay raw: 4 registers each
  bf16x8 wq8, wk8;
  if (norm) {
    wq8 = *reinterpret_cast<const bf16x8*>(qw + ln.e0);
    wk8 = *reinterpret_cast<const bf16x8*>(kw + ln.e0);
  }
  const float sg = ln.first ? -1.f : 1.f;  // first half: x1 c - x2 s;  second half: x2 c + x1 s
  const bf16* src = qkv + (int64_t)tok * ldqkv + ln.e0;
  for (int hb = 0; hb < H; hb += L::HPW * UNR) {
    bf16x8 raw[UNR];
#pragma unroll
    for (int u = 0; u < UNR; ++u) {
      const int h = hb + u * L::HPW + ln.sub;
      if (h < H)
        raw[u] = *reinterpret_cast<const bf16x8*>(
            src + (h < Hq ? (int64_t)h * qstride : (int64_t)Hq * qstride + (int64_t)(h - Hq) * D));
      else
        raw[u] = bf16x8{};
    }
#pragma unroll
    for (int u = 0; u < UNR; ++u) {
      const int h = hb + u * L::HPW + ln.sub;
      const bool is_q = h < Hq;
      float f[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 t = __bfloat1622float2(raw[u].h[i]);
        f[2 * i] = t.x;
        f[2 * i + 1] = t.y;
      }
      float r = 1.f;
      if (norm) {
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) ss += f[i] * f[i];
#pragma unroll
        for (int o = L::LPH / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        r = rsqrtf(ss / (float)D + eps);
        const bf16x8& w8 = is_q ? wq8 : wk8;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 t = __bfloat1622float2(w8.h[i]);
          f[2 * i] *= r * t.x;
          f[2 * i + 1] *= r * t.y;
        }
      }
      float px[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) px[i] = __shfl_sync(0xffffffffu, f[i], ln.partner);
      if (ln.roped)
#pragma unroll
        for (int i = 0; i < 8; ++i) f[i] = f[i] * c[i] + sg * px[i] * sn[i];
      if (h < H) {
        if (ln.e0 == 0) rstd[(int64_t)tok * H + h] = r;
        bf16* dst = is_q ? (q + ((int64_t)tok * Hq + h) * D) : (k + ((int64_t)tok * Hkv + (h - Hq)) * D);
        store8(dst + ln.e0, f);
      }
    }
  }
}

template <int D>
__global__ void __launch_bounds__(256) qk_norm_rope_bwd_vec_kernel(
    const bf16* __restrict__ dq, const bf16* __restrict__ dk, const bf16* __restrict__ qkv, int64_t ldqkv,
    const bf16* __restrict__ qw, const bf16* __restrict__ kw, const float* __restrict__ cos_t,
    const float* __restrict__ sin_t, const int* __restrict__ pos, const float* __restrict__ rstd,
    bf16* __restrict__ dqkv, int64_t lddqkv, float* __restrict__ dqw, float* __restrict__ dkw, int M, int Hq,
    int Hkv, int rd, int qstride) {
  using L = QkLane<D>;
  constexpr int UNR = 2;
  __shared__ float sred[8][2][D];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const L ln(lane, rd);
  const int H = Hq + Hkv, half = rd >> 1;
  float wq[8], wk[8], accq[8], acck[8];
  load8(qw + ln.e0, wq);
  load8(kw + ln.e0, wk);
#pragma unroll
  for (int i = 0; i < 8; ++i) accq[i] = acck[i] = 0.f;
  const float sg = ln.first ? 1.f : -1.f;  // inverse rotation: dn1 = g1 c + g2 s,  dn2 = g2 c - g1 s
  for (int tok = blockIdx.x * (blockDim.x >> 5) + warp; tok < M; tok += gridDim.x * (blockDim.x >> 5)) {
    float c[8], sn[8];
    if (ln.roped) load_rope8(cos_t, sin_t, (int64_t)pos[tok] * half + (ln.first ? ln.e0 : ln.e0 - half), c, sn);
    const bf16* xrow = qkv + (int64_t)tok * ldqkv + ln.e0;
    bf16* orow = dqkv + (int64_t)tok * lddqkv + ln.e0;
    for (int hb = 0; hb < H; hb += L::HPW * UNR) {
      float g[UNR][8], xs[UNR][8], r[UNR];
#pragma unroll
      for (int u = 0; u < UNR; ++u) {
        const int h = hb + u * L::HPW + ln.sub;
        if (h < H) {
          const bool is_q = h < Hq;
          load8((is_q ? dq + ((int64_t)tok * Hq + h) * D : dk + ((int64_t)tok * Hkv + (h - Hq)) * D) + ln.e0, g[u]);
          load8(xrow + (is_q ? (int64_t)h * qstride : (int64_t)Hq * qstride + (int64_t)(h - Hq) * D), xs[u]);
          r[u] = rstd[(int64_t)tok * H + h];
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) g[u][i] = xs[u][i] = 0.f;
          r[u] = 0.f;
        }
      }
#pragma unroll
      for (int u = 0; u < UNR; ++u) {
        const int h = hb + u * L::HPW + ln.sub;
        const bool is_q = h < Hq;
        float pg[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) pg[i] = __shfl_sync(0xffffffffu, g[u][i], ln.partner);
        if (ln.roped)
#pragma unroll
          for (int i = 0; i < 8; ++i) g[u][i] = g[u][i] * c[i] + sg * pg[i] * sn[i];
        float dot = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          xs[u][i] *= r[u];  // xhat
          dot += g[u][i] * (is_q ? wq[i] : wk[i]) * xs[u][i];
        }
#pragma unroll
        for (int o = L::LPH / 2; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
        dot /= (float)D;
        if (h < H) {
          float o[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            o[i] = r[u] * (g[u][i] * (is_q ? wq[i] : wk[i]) - xs[u][i] * dot);
            const float t = g[u][i] * xs[u][i];
            if (is_q) accq[i] += t; else acck[i] += t;
          }
          store8(orow + (is_q ? (int64_t)h * qstride : (int64_t)Hq * qstride + (int64_t)(h - Hq) * D), o);
        }
      }
    }
  }
  // the head groups of a warp own the same columns: fold them, then the warps, then global
#pragma unroll
  for (int o = L::LPH; o < 32; o <<= 1)
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      accq[i] += __shfl_xor_sync(0xffffffffu, accq[i], o);
      acck[i] += __shfl_xor_sync(0xffffffffu, acck[i], o);
    }
  if (ln.sub == 0)
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      sred[warp][0][ln.e0 + i] = accq[i];
      sred[warp][1][ln.e0 + i] = acck[i];
    }
  __syncthreads();
  const int nw = blockDim.x >> 5;
  for (int e = threadIdx.x; e < 2 * D; e += blockDim.x) {
    float t = 0.f;
    for (int wi = 0; wi < nw; ++wi) t += sred[wi][e / D][e % D];
    float* dst = e < D ? (dqw ? dqw + e : nullptr) : (dkw ? dkw + (e - D) : nullptr);
    if (dst) atomicAdd(dst, t);
  }
}

static bool qk_vec_ok(int d, int rd, int64_t ldqkv, int qstride, std::initializer_list<const void*> ptrs) {
  if (!(d == 64 || d == 128 || d == 256) || rd % 16 != 0 || rd > d || ldqkv % 8 != 0 || qstride % 8 != 0)
    return false;
  for (const void* p : ptrs)
    if (p != nullptr && !aligned16(p)) return false;
  return true;
}

void qk_norm_rope_fwd(const bf16* qkv, int64_t ldqkv, const bf16* qw, const bf16* kw, const float* cos_t,
                      const float* sin_t, const int* pos, bf16* q, bf16* k, float* rstd, int M, int Hq,
                      int Hkv, int d, int rd, float eps, int qstride, cudaStream_t s) {
  const int warps = 8;
  const int64_t total = (int64_t)M * (Hq + Hkv);
  if (qk_vec_ok(d, rd, ldqkv, qstride, {qkv, qw, kw, cos_t, sin_t, q, k})) {
    const int blocks = ceil_div(M, warps);  // one warp per token
#define TRIDA_QK_FWD(DD)                                                                                  \
  qk_norm_rope_fwd_vec_kernel<DD><<<blocks, warps * 32, 0, s>>>(qkv, ldqkv, qw, kw, cos_t, sin_t, pos, q, k, \
                                                                rstd, M, Hq, Hkv, rd, eps, qstride)
    if (d == 64) TRIDA_QK_FWD(64); else if (d == 128) TRIDA_QK_FWD(128); else TRIDA_QK_FWD(256);
#undef TRIDA_QK_FWD
    return;
  }
  qk_norm_rope_fwd_kernel<<<ceil_div(total, warps), warps * 32, 0, s>>>(qkv, ldqkv, qw, kw, cos_t, sin_t, pos,
                                                                       q, k, rstd, M, Hq, Hkv, d, rd, eps, qstride);
}

void qk_norm_rope_bwd(const bf16* dq, const bf16* dk, const bf16* qkv, int64_t ldqkv, const bf16* qw,
                      const bf16* kw, const float* cos_t, const float* sin_t, const int* pos,
                      const float* rstd, bf16* dqkv, int64_t lddqkv, float* dqw, float* dkw, int M, int Hq,
                      int Hkv, int d, int rd, int qstride, int sm_count, cudaStream_t s) {
  const int warps = 8;
  const int64_t total = (int64_t)M * (Hq + Hkv);
  if (qk_vec_ok(d, rd, ldqkv, qstride, {dq, dk, qkv, qw, kw, cos_t, sin_t, dqkv}) && lddqkv % 8 == 0) {
    int64_t blocks = ceil_div(M, warps * 4);  // one warp per token, about 4 tokens a warp
    blocks = blocks > sm_count * 6 ? sm_count * 6 : blocks;
#define TRIDA_QK_BWD(DD)                                                                                   \
  qk_norm_rope_bwd_vec_kernel<DD><<<(int)blocks, warps * 32, 0, s>>>(dq, dk, qkv, ldqkv, qw, kw, cos_t, sin_t, \
                                                                     pos, rstd, dqkv, lddqkv, dqw, dkw, M, Hq,  \
                                                                     Hkv, rd, qstride)
    if (d == 64) TRIDA_QK_BWD(64); else if (d == 128) TRIDA_QK_BWD(128); else TRIDA_QK_BWD(256);
#undef TRIDA_QK_BWD
    return;
  }
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
