// Serving kernels for the self-speculative decode step (sm_100a).
//
// A decode step runs one forward over a "canvas" of blk rows per active request: the first n_clean
// rows are token-causal, the remaining (MASK) rows see the whole canvas; every row sees the whole
// cached prefix.  Behaviour follows the reference's canvas rule
// (inference/zoro-1/mlx/trida_mlx/model.py:461-470, SGLang/vLLM self-spec backends) and its commit
// (model.py:486-507): the KV of the first `adv` canvas rows stays, the gated-delta state advances
// by `adv` rows and the conv window becomes the last K-1 pre-conv rows.
//
//   canvas_attn   split-K decode attention: CTA = 64 query rows (the GQA group's heads x canvas
//                 rows of one request) x one 256-key slice of that request's [prefix ; canvas]
//                 keys; mma.sync bf16 tiles, online softmax; a combine pass merges the slices.
//   kv_append     writes the canvas rows' K (post norm/RoPE) and V into the slot's cache rows.
//   canvas_conv   depthwise conv + SiLU over [cached window ; canvas rows].
//   conv_commit   new window = last K-1 rows of [window ; first adv canvas rows].
//   argmax_rows   greedy token per logits row.
//   conf_argmax_rows  greedy token, row max and softmax normaliser per row (denoise gate).
#include <cfloat>

#include "common.cuh"
#include "ops.h"
#include "warp_mma.cuh"

namespace trida {
namespace serve {

using namespace attn;

struct CanvasAttnParams {
  const bf16* q;          // [B*blk, Hq, D]
  const bf16* kc;         // [slots, maxlen, Hkv, D]
  const bf16* vc;
  const int* slot;        // [B]
  const int* pos;         // [B] cached prefix length (canvas keys start here)
  const int* ptab;        // paged cache: [slots, maxpages] page of every 64 positions (kc / vc are
                          // [pages, 64, Hkv, D]); null: dense [slots, maxlen, Hkv, D] cache
  int maxpages;
  float* po;              // [B, nsplit, Hq, blk, D] partial outputs (unnormalised)
  float* pm;              // [B, nsplit, Hq, blk] running max (scaled, log2 domain)
  float* pl;              // [B, nsplit, Hq, blk] running sum
  int blk, n_clean, Hq, Hkv, maxlen, nsplit, ks;
  float scale_log2;
};

template <int D>
__global__ void __launch_bounds__(128) canvas_attn_kernel(const CanvasAttnParams p) {
  constexpr int BM = 64, BN = 64, NT = 128;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  bf16* sQ = reinterpret_cast<bf16*>(smem_raw);
  bf16* sK = sQ + BM * D;
  bf16* sV = sK + 2 * BN * D;
  const int split = blockIdx.x, b = blockIdx.z;
  const int G = p.Hq / p.Hkv;
  const int nqt = (G * p.blk + BM - 1) / BM;
  const int qtile = blockIdx.y % nqt, hk = blockIdx.y / nqt;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int slot = p.slot[b], pos = p.pos[b];
  const int kend = pos + p.blk;
  const int k0 = split * p.ks, k1 = min(kend, k0 + p.ks);
  const int nrows = G * p.blk;

  // gather the tile's query rows: row r -> (head hk*G + r / blk, canvas row r % blk)
  for (int c = threadIdx.x; c < BM * D / 8; c += NT) {
    const int row = c / (D / 8), col = (c % (D / 8)) * 8;
    const int qr = qtile * BM + row;
    const bool ok = qr < nrows;
    const int g = ok ? qr / p.blk : 0, i = ok ? qr % p.blk : 0;
    const bf16* src = p.q + ((int64_t)(b * p.blk + i) * p.Hq + hk * G + g) * D + col;
    cp_async16(sQ + swz<D>(row, col), src, ok);
  }
  const int64_t ktok = (int64_t)p.Hkv * D;
  const int ntile = k1 > k0 ? (k1 - k0 + BN - 1) / BN : 0;
  // first key row of tile `it` (a 64-key tile is exactly one page of a paged cache)
  auto key_row = [&](int it) -> int64_t {
    const int kp = k0 + it * BN;
    if (p.ptab != nullptr) return ((int64_t)p.ptab[(int64_t)slot * p.maxpages + kp / BN] * BN) * ktok + hk * D;
    return ((int64_t)slot * p.maxlen + kp) * ktok + hk * D;
  };
  auto issue_kv = [&](int it) {
    const int buf = it & 1;
    const int64_t r0 = key_row(it);
    load_tile<D, BN, NT>(sK + buf * BN * D, p.kc + r0, ktok, 0, k1 - k0 - it * BN);
    load_tile<D, BN, NT>(sV + buf * BN * D, p.vc + r0, ktok, 0, k1 - k0 - it * BN);
  };
  if (ntile > 0) issue_kv(0);
  cp_async_commit();

  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_i[2] = {-INFINITY, -INFINITY}, l_i[2] = {0.f, 0.f};
  const int wr = warp * 16;
  const int r_lo = wr + (lane >> 2), r_hi = r_lo + 8;
  const int qlo = qtile * BM + r_lo, qhi = qtile * BM + r_hi;
  const int ilo = qlo % p.blk, ihi = qhi % p.blk;     // canvas row of each query row

  for (int it = 0; it < ntile; ++it) {
    if (it + 1 < ntile) issue_kv(it + 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const int buf = it & 1;
    const bf16* cK = sK + buf * BN * D;
    const bf16* cV = sV + buf * BN * D;
    float s[BN / 8][4];
#pragma unroll
    for (int j = 0; j < BN / 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t qa[4];
      {
        const int row = wr + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int col = kk * 16 + (lane >> 4) * 8;
        ldsm_x4(qa, sQ + swz<D>(row, col));
      }
#pragma unroll
      for (int jp = 0; jp < BN / 16; ++jp) {
        uint32_t bfr[4];
        const int row = jp * 16 + (lane & 7) + (lane >> 4) * 8;
        const int col = kk * 16 + ((lane >> 3) & 1) * 8;
        ldsm_x4(bfr, cK + swz<D>(row, col));
        mma16816(s[2 * jp], qa, bfr[0], bfr[1]);
        mma16816(s[2 * jp + 1], qa, bfr[2], bfr[3]);
      }
    }
    // mask: keys beyond the canvas; canvas key c visible to canvas row i iff c <= i or i >= n_clean
#pragma unroll
    for (int j = 0; j < BN / 8; ++j) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int kj = k0 + it * BN + j * 8 + (lane & 3) * 2 + e;
        const int c = kj - pos;
        const bool in = kj < k1;
        const bool alo = in && (c < 0 || c <= ilo || ilo >= p.n_clean);
        const bool ahi = in && (c < 0 || c <= ihi || ihi >= p.n_clean);
        if (!alo) s[j][e] = -INFINITY;
        if (!ahi) s[j][2 + e] = -INFINITY;
      }
    }
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < BN / 8; ++j) {
      mx[0] = fmaxf(mx[0], fmaxf(s[j][0], s[j][1]));
      mx[1] = fmaxf(mx[1], fmaxf(s[j][2], s[j][3]));
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
    }
    float alpha[2], mref[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const float mnew = fmaxf(m_i[r], mx[r]);
      mref[r] = (mnew == -INFINITY) ? 0.f : mnew * p.scale_log2;
      alpha[r] = (m_i[r] == -INFINITY) ? 0.f : exp2f(m_i[r] * p.scale_log2 - mref[r]);
      m_i[r] = mnew;
    }
    float rs[2] = {0.f, 0.f};
    uint32_t pf[BN / 16][4];
#pragma unroll
    for (int j = 0; j < BN / 8; ++j) {
      const float p0 = exp2f(s[j][0] * p.scale_log2 - mref[0]);
      const float p1 = exp2f(s[j][1] * p.scale_log2 - mref[0]);
      const float p2 = exp2f(s[j][2] * p.scale_log2 - mref[1]);
      const float p3 = exp2f(s[j][3] * p.scale_log2 - mref[1]);
      rs[0] += p0 + p1;
      rs[1] += p2 + p3;
      pf[j >> 1][(j & 1) * 2 + 0] = pack_bf16(p0, p1);
      pf[j >> 1][(j & 1) * 2 + 1] = pack_bf16(p2, p3);
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) l_i[r] = l_i[r] * alpha[r] + rs[r];
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      o[i][0] *= alpha[0];
      o[i][1] *= alpha[0];
      o[i][2] *= alpha[1];
      o[i][3] *= alpha[1];
    }
#pragma unroll
    for (int kk = 0; kk < BN / 16; ++kk) {
#pragma unroll
      for (int dp = 0; dp < D / 16; ++dp) {
        uint32_t bfr[4];
        const int row = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int col = dp * 16 + (lane >> 4) * 8;
        ldsm_x4_t(bfr, cV + swz<D>(row, col));
        mma16816(o[2 * dp], pf[kk], bfr[0], bfr[1]);
        mma16816(o[2 * dp + 1], pf[kk], bfr[2], bfr[3]);
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    float l = l_i[r];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    l_i[r] = l;
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int qr = r ? qhi : qlo;
    if (qr >= nrows) continue;
    const int g = qr / p.blk, i = qr % p.blk;
    const int h = hk * G + g;
    const int64_t ri = (((int64_t)b * p.nsplit + split) * p.Hq + h) * p.blk + i;
    float* dst = p.po + ri * D;
#pragma unroll
    for (int t = 0; t < D / 8; ++t) {
      const int col = t * 8 + (lane & 3) * 2;
      *reinterpret_cast<float2*>(dst + col) = make_float2(o[t][2 * r], o[t][2 * r + 1]);
    }
    if ((lane & 3) == 0) {
      p.pm[ri] = m_i[r] == -INFINITY ? -INFINITY : m_i[r] * p.scale_log2;
      p.pl[ri] = l_i[r];
    }
  }
}

// out[b*blk + i, h, :] = sum_s 2^(m_s - M) o_s / sum_s 2^(m_s - M) l_s   (one warp per row)
__global__ void canvas_combine_kernel(const float* po, const float* pm, const float* pl, bf16* out, int B, int nsplit,
                                      int Hq, int blk, int D) {
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= (int64_t)B * Hq * blk) return;
  const int b = (int)(gw / (Hq * blk));
  const int h = (int)((gw / blk) % Hq), i = (int)(gw % blk);
  float M = -INFINITY;
  for (int s = 0; s < nsplit; ++s) M = fmaxf(M, pm[(((int64_t)b * nsplit + s) * Hq + h) * blk + i]);
  float L = 0.f;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int s = 0; s < nsplit; ++s) {
    const int64_t ri = (((int64_t)b * nsplit + s) * Hq + h) * blk + i;
    const float m = pm[ri];
    if (m == -INFINITY) continue;
    const float w = exp2f(m - M);
    L += w * pl[ri];
    for (int c = lane, e = 0; c < D; c += 32, ++e) acc[e] += w * po[ri * D + c];
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  bf16* dst = out + ((int64_t)(b * blk + i) * Hq + h) * D;
  for (int c = lane, e = 0; c < D; c += 32, ++e) dst[c] = __float2bfloat16(acc[e] * inv);
}

// cache[slot, pos + i] <- k / v of canvas row i (k: [B*blk, Hkv, D] contiguous; v: row-strided)
__global__ void kv_append_kernel(const bf16* k, const bf16* v, int64_t ldv, bf16* kc, bf16* vc, const int* slot,
                                 const int* pos, int B, int blk, int Hkv, int D, int maxlen, const int* ptab,
                                 int maxpages) {
  const int64_t n8 = (int64_t)B * blk * Hkv * D / 8;
  for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < n8; g += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = g * 8;
    const int64_t row = e / (Hkv * D);
    const int rem = (int)(e % (Hkv * D));
    const int b = (int)(row / blk), i = (int)(row % blk);
    const int p = pos[b] + i;
    if (p >= maxlen) continue;
    const int64_t crow = ptab != nullptr ? (int64_t)ptab[(int64_t)slot[b] * maxpages + p / 64] * 64 + p % 64
                                         : (int64_t)slot[b] * maxlen + p;
    const int64_t dst = crow * Hkv * D + rem;
    *reinterpret_cast<uint4*>(kc + dst) = *reinterpret_cast<const uint4*>(k + row * Hkv * D + rem);
    *reinterpret_cast<uint4*>(vc + dst) = *reinterpret_cast<const uint4*>(v + row * ldv + rem);
  }
}

// y[b*blk + j, c] = silu(sum_tap w[c, tap] x(j - (K-1-tap))), x(i < 0) from the slot's window
__global__ void canvas_conv_kernel(const bf16* x, int64_t ldx, const bf16* win, const bf16* w, bf16* y, int64_t ldy,
                                   const int* slot, int B, int blk, int C, int K) {
  const int64_t n = (int64_t)B * blk * (C / 8);
  for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < n; g += (int64_t)gridDim.x * blockDim.x) {
    const int c8 = (int)(g % (C / 8)) * 8;
    const int64_t row = g / (C / 8);
    const int b = (int)(row / blk), j = (int)(row % blk);
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int tap = 0; tap < K; ++tap) {
      const int src = j - (K - 1 - tap);
      float xv[8];
      if (src >= 0) load8(x + ((int64_t)b * blk + src) * ldx + c8, xv);
      else load8(win + ((int64_t)slot[b] * (K - 1) + (K - 1 + src)) * C + c8, xv);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = fmaf(__bfloat162float(w[(c8 + e) * K + tap]), xv[e], acc[e]);
    }
    float out[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) out[e] = acc[e] / (1.f + expf(-acc[e]));
    store8(y + row * ldy + c8, out);
  }
}

// The same canvas convolution for the 4-tap kernel of the models served here: a thread owns 8
// channels of a 16-row tile, loads its 32 weights once (one 64-byte run of the [C][4] weight) and
// keeps the three previous input rows in registers, so each input row is read once per tile
// instead of once per tap.
constexpr int CONV4_ROWS = 16;
__global__ void canvas_conv4_kernel(const bf16* __restrict__ x, int64_t ldx, const bf16* __restrict__ win,
                                    const bf16* __restrict__ w, bf16* __restrict__ y, int64_t ldy,
                                    const int* __restrict__ slot, int B, int blk, int C) {
  const int C8 = C / 8;
  const int tiles = (blk + CONV4_ROWS - 1) / CONV4_ROWS;
  const int64_t n = (int64_t)B * tiles * C8;
  for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < n; g += (int64_t)gridDim.x * blockDim.x) {
    const int c8 = (int)(g % C8) * 8;
    const int64_t rest = g / C8;
    const int tile = (int)(rest % tiles), b = (int)(rest / tiles);
    const int j0 = tile * CONV4_ROWS, j1 = min(blk, j0 + CONV4_ROWS);
    float wt[8][4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {          // 32 consecutive bf16: channel c8 + 2q, c8 + 2q + 1 x 4 taps
      float f[8];
      load8(w + (int64_t)c8 * 4 + q * 8, f);
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        wt[2 * q][t] = f[t];
        wt[2 * q + 1][t] = f[4 + t];
      }
    }
    float h[3][8];                          // input rows j - 3, j - 2, j - 1
#pragma unroll
    for (int t = 0; t < 3; ++t) {
      const int src = j0 - 3 + t;
      if (src >= 0) load8(x + ((int64_t)b * blk + src) * ldx + c8, h[t]);
      else load8(win + ((int64_t)slot[b] * 3 + (3 + src)) * C + c8, h[t]);
    }
    // the rows' loads do not depend on each other: unrolled, several are in flight at once
#pragma unroll 4
    for (int j = j0; j < j1; ++j) {
      float xv[8], out[8];
      load8(x + ((int64_t)b * blk + j) * ldx + c8, xv);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float acc = 0.f;
        acc = fmaf(wt[e][0], h[0][e], acc);
        acc = fmaf(wt[e][1], h[1][e], acc);
        acc = fmaf(wt[e][2], h[2][e], acc);
        acc = fmaf(wt[e][3], xv[e], acc);
        out[e] = __fdividef(acc, 1.f + __expf(fminf(-acc, 80.f)));   // SiLU (fast exp / divide)
      }
      store8(y + ((int64_t)b * blk + j) * ldy + c8, out);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        h[0][e] = h[1][e];
        h[1][e] = h[2][e];
        h[2][e] = xv[e];
      }
    }
  }
}

// window[slot] <- last K-1 rows of [window ; x rows 0..adv-1] (rows of entry b at x + b*rows_per*ldx)
__global__ void conv_commit_kernel(const bf16* x, int64_t ldx, int rows_per, bf16* win, const int* slot,
                                   const int* adv, int B, int C, int K) {
  const int64_t n = (int64_t)B * (C / 8);
  for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < n; g += (int64_t)gridDim.x * blockDim.x) {
    const int c8 = (int)(g % (C / 8)) * 8;
    const int b = (int)(g / (C / 8));
    const int a = adv[b];
    bf16* wb = win + (int64_t)slot[b] * (K - 1) * C + c8;
    uint4 nw[3];
    for (int r = 0; r < K - 1 && r < 3; ++r) {
      const int idx = a + r;     // index into [window (K-1 rows) ; x rows]
      nw[r] = idx < K - 1 ? *reinterpret_cast<const uint4*>(wb + (int64_t)idx * C)
                          : *reinterpret_cast<const uint4*>(x + ((int64_t)b * rows_per + idx - (K - 1)) * ldx + c8);
    }
    for (int r = 0; r < K - 1 && r < 3; ++r) *reinterpret_cast<uint4*>(wb + (int64_t)r * C) = nw[r];
  }
}

// out[r] = argmax_v logits[r, v] (first index on ties); one CTA per row
__global__ void argmax_rows_kernel(const float* logits, int64_t ld, int V, int64_t* out) {
  const float* row = logits + (int64_t)blockIdx.x * ld;
  float best = -INFINITY;
  int idx = 0x7fffffff;
  for (int v = threadIdx.x; v < V; v += blockDim.x) {
    const float x = row[v];
    if (x > best) { best = x; idx = v; }
  }
  __shared__ float sb[32];
  __shared__ int si[32];
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ob > best || (ob == best && oi < idx)) { best = ob; idx = oi; }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { sb[warp] = best; si[warp] = idx; }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    best = lane < nw ? sb[lane] : -INFINITY;
    idx = lane < nw ? si[lane] : 0x7fffffff;
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
      if (ob > best || (ob == best && oi < idx)) { best = ob; idx = oi; }
    }
    if (lane == 0) out[blockIdx.x] = idx;
  }
}

// Per logits row: first argmax, row max and sum(exp(x - max)) -- the greedy token and its softmax
// probability (1 / sum) in one pass; with vocabulary-parallel shards the host combines (max, sum)
// pairs across ranks.  Row r lives at logits + (r / rpb) * sb + (r % rpb) * ld.  One CTA per row.
__global__ void conf_argmax_rows_kernel(const float* logits, int rpb, int64_t sb, int64_t ld, int V,
                                        int64_t* out_idx, float* out_max, float* out_sum) {
  const int r = blockIdx.x;
  const float* row = logits + (int64_t)(r / rpb) * sb + (int64_t)(r % rpb) * ld;
  float m = -INFINITY, z = 0.f;
  int idx = 0x7fffffff;
  for (int v = threadIdx.x; v < V; v += blockDim.x) {
    const float x = row[v];
    if (x > m) {
      z = z * __expf(m - x) + 1.f;
      m = x;
      idx = v;
    } else {
      z += __expf(x - m);
    }
  }
  auto merge = [](float& m1, float& z1, int& i1, float m2, float z2, int i2) {
    if (m2 > m1 || (m2 == m1 && i2 < i1)) {
      z1 = z2 + (m1 == -INFINITY ? 0.f : z1 * __expf(m1 - m2));
      m1 = m2;
      i1 = i2;
    } else {
      z1 += (m2 == -INFINITY ? 0.f : z2 * __expf(m2 - m1));
    }
  };
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, m, o);
    const float oz = __shfl_xor_sync(0xffffffffu, z, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    merge(m, z, idx, om, oz, oi);
  }
  __shared__ float sm[32], sz[32];
  __shared__ int si[32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { sm[warp] = m; sz[warp] = z; si[warp] = idx; }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    m = lane < nw ? sm[lane] : -INFINITY;
    z = lane < nw ? sz[lane] : 0.f;
    idx = lane < nw ? si[lane] : 0x7fffffff;
    for (int o = 16; o > 0; o >>= 1) {
      const float om = __shfl_xor_sync(0xffffffffu, m, o);
      const float oz = __shfl_xor_sync(0xffffffffu, z, o);
      const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
      merge(m, z, idx, om, oz, oi);
    }
    if (lane == 0) {
      out_idx[r] = idx;
      out_max[r] = m;
      out_sum[r] = z;
    }
  }
}

template <int D>
size_t canvas_smem() { return (size_t)(64 * D + 4 * 64 * D) * 2; }

}  // namespace serve

int canvas_attention(const bf16* q, const bf16* kc, const bf16* vc, const int* slot, const int* pos, bf16* out,
                     float* work, int B, int blk, int n_clean, int Hq, int Hkv, int D, int maxlen, int max_keys,
                     float scale, cudaStream_t s, const int* ptab, int maxpages) {
  using namespace serve;
  CanvasAttnParams p;
  p.q = q; p.kc = kc; p.vc = vc; p.slot = slot; p.pos = pos; p.ptab = ptab; p.maxpages = maxpages;
  p.blk = blk; p.n_clean = n_clean; p.Hq = Hq; p.Hkv = Hkv; p.maxlen = maxlen;
  p.ks = 256;
  p.nsplit = (max_keys + p.ks - 1) / p.ks;
  const int64_t rows = (int64_t)B * p.nsplit * Hq * blk;
  p.po = work; p.pm = work + rows * D; p.pl = p.pm + rows;
  p.scale_log2 = scale * 1.44269504088896340736f;
  const int G = Hq / Hkv;
  const int nqt = (G * blk + 63) / 64;
  dim3 grid(p.nsplit, nqt * Hkv, B);
  switch (D) {
    case 128: {
      static bool init = false;
      if (!init) { cudaFuncSetAttribute(canvas_attn_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)canvas_smem<128>()); init = true; }
      canvas_attn_kernel<128><<<grid, 128, canvas_smem<128>(), s>>>(p);
      break;
    }
    case 256: {
      static bool init = false;
      if (!init) { cudaFuncSetAttribute(canvas_attn_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)canvas_smem<256>()); init = true; }
      canvas_attn_kernel<256><<<grid, 128, canvas_smem<256>(), s>>>(p);
      break;
    }
    default: return -1;
  }
  const int64_t warps = (int64_t)B * Hq * blk;
  canvas_combine_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, s>>>(p.po, p.pm, p.pl, out, B, p.nsplit, Hq,
                                                                            blk, D);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

void canvas_combine(const float* po, const float* pm, const float* pl, bf16* out, int B, int nsplit, int Hq, int blk,
                    int D, cudaStream_t s) {
  const int64_t warps = (int64_t)B * Hq * blk;
  serve::canvas_combine_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, s>>>(po, pm, pl, out, B, nsplit, Hq,
                                                                                   blk, D);
}

int64_t canvas_work_floats(int B, int blk, int Hq, int D, int max_keys) {
  const int nsplit = (max_keys + 255) / 256;
  const int64_t rows = (int64_t)B * nsplit * Hq * blk;
  return rows * D + 2 * rows;
}

void kv_append(const bf16* k, const bf16* v, int64_t ldv, bf16* kc, bf16* vc, const int* slot, const int* pos, int B,
               int blk, int Hkv, int D, int maxlen, cudaStream_t s, const int* ptab, int maxpages) {
  const int64_t n8 = (int64_t)B * blk * Hkv * D / 8;
  const int blocks = (int)std::min<int64_t>((n8 + 255) / 256, 4096);
  serve::kv_append_kernel<<<blocks, 256, 0, s>>>(k, v, ldv, kc, vc, slot, pos, B, blk, Hkv, D, maxlen, ptab, maxpages);
}

void canvas_conv(const bf16* x, int64_t ldx, const bf16* win, const bf16* w, bf16* y, int64_t ldy, const int* slot,
                 int B, int blk, int C, int K, cudaStream_t s) {
  if (K == 4 && C % 8 == 0 && ldx % 8 == 0 && ldy % 8 == 0) {
    const int64_t n4 = (int64_t)B * ((blk + serve::CONV4_ROWS - 1) / serve::CONV4_ROWS) * (C / 8);
    const int blocks = (int)std::min<int64_t>((n4 + 255) / 256, 8192);
    serve::canvas_conv4_kernel<<<blocks, 256, 0, s>>>(x, ldx, win, w, y, ldy, slot, B, blk, C);
    return;
  }
  const int64_t n = (int64_t)B * blk * (C / 8);
  const int blocks = (int)std::min<int64_t>((n + 255) / 256, 8192);
  serve::canvas_conv_kernel<<<blocks, 256, 0, s>>>(x, ldx, win, w, y, ldy, slot, B, blk, C, K);
}

void conv_commit(const bf16* x, int64_t ldx, int rows_per, bf16* win, const int* slot, const int* adv, int B, int C,
                 int K, cudaStream_t s) {
  const int64_t n = (int64_t)B * (C / 8);
  const int blocks = (int)std::min<int64_t>((n + 255) / 256, 4096);
  serve::conv_commit_kernel<<<blocks, 256, 0, s>>>(x, ldx, rows_per, win, slot, adv, B, C, K);
}

void argmax_rows(const float* logits, int64_t ld, int rows, int V, int64_t* out, cudaStream_t s) {
  serve::argmax_rows_kernel<<<rows, 1024, 0, s>>>(logits, ld, V, out);
}

void conf_argmax_rows(const float* logits, int rows, int rpb, int64_t sb, int64_t ld, int V, int64_t* idx,
                      float* mx, float* sum, cudaStream_t s) {
  if (rows > 0) serve::conf_argmax_rows_kernel<<<rows, 1024, 0, s>>>(logits, rpb, sb, ld, V, idx, mx, sum);
}

}  // namespace trida
