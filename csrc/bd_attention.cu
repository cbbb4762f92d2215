// Block-diffusion attention, forward and backward, for sm_100a.
//
// The mask is never materialised.  Every token carries a 16-byte metadata word
//   {opos, rblk, segid, seg | view << 8}
// (original position, response block, packed-document id, segment class PAD/SHARED/XT/X0 and the
// complementary-view id) and the rule of the reference's flex mask_mod
// (train/models/block_diffusion.py:245-264, packed :312-328, merged views :344-361) is evaluated
// from two such words.  A classification pass labels each 64x64 (query, key) tile EMPTY / FULL /
// PARTIAL exactly; the attention kernels walk only non-empty tiles from compacted per-tile lists
// and evaluate the per-element rule only on PARTIAL tiles.
//
// Math path of this version: warp-level bf16 MMA (m16n8k16) with fp32 accumulation, online
// softmax in registers (exp2 domain), K/V double-buffered through shared memory with cp.async
// and an XOR swizzle so ldmatrix is bank-conflict free.  GQA: query head h reads KV head
// h / (Hq / Hkv).
#include "common.cuh"
#include "ops.h"
#include "warp_mma.cuh"

#include <cfloat>
#include <climits>

namespace trida {
namespace attn {

constexpr int SEG_PAD = 0, SEG_SHARED = 1, SEG_XT = 2, SEG_X0 = 3;
constexpr int FLAG_X0_TOKEN_CAUSAL = 1, FLAG_WITHIN_BLOCK_CAUSAL = 2;
constexpr int TILE = 64;  // classification granularity (queries x keys)
constexpr int CLS_EMPTY = 0, CLS_FULL = 1, CLS_PARTIAL = 2;

__device__ __forceinline__ bool allowed(const int4 q, const int4 k, bool same_index, int flags) {
  if (same_index) return true;
  const int sq = q.w & 0xff, sk = k.w & 0xff;
  if (sk == SEG_PAD || q.z != k.z) return false;
  const int vq = q.w >> 8, vk = k.w >> 8;
  bool r = (sk == SEG_SHARED) & (k.x <= q.x);
  r |= (sq == SEG_XT) & (sk == SEG_XT) & (q.y == k.y) & (vq == vk) &
       (!(flags & FLAG_WITHIN_BLOCK_CAUSAL) || (k.x <= q.x));
  r |= (sq == SEG_XT) & (sk == SEG_X0) & (k.y < q.y);
  r |= (sq == SEG_X0) & (sk == SEG_X0) &
       ((flags & FLAG_X0_TOKEN_CAUSAL) ? (k.x <= q.x) : (k.y <= q.y));
  return r;
}

__device__ __forceinline__ int4 load_meta(const int4* meta, int b, int T, int i) {
  if (i < T) return meta[(int64_t)b * T + i];
  return make_int4(INT_MAX, INT_MAX, -2, SEG_PAD);
}

// ---- classification: one CTA per (key tile, query tile, batch) -----------------------------
__global__ void classify_kernel(const int4* __restrict__ meta, int T, int flags, uint8_t* __restrict__ cls) {
  __shared__ int4 mq[TILE], mk[TILE];
  const int kt = blockIdx.x, qt = blockIdx.y, b = blockIdx.z;
  const int nt = gridDim.x;
  if (threadIdx.x < TILE) mq[threadIdx.x] = load_meta(meta, b, T, qt * TILE + threadIdx.x);
  else if (threadIdx.x < 2 * TILE) mk[threadIdx.x - TILE] = load_meta(meta, b, T, kt * TILE + threadIdx.x - TILE);
  __syncthreads();
  int any = 0, all = 1;
  for (int e = threadIdx.x; e < TILE * TILE; e += blockDim.x) {
    const int i = e / TILE, j = e % TILE;
    const int qi = qt * TILE + i, kj = kt * TILE + j;
    const bool in = (qi < T) && (kj < T);
    const bool a = in && allowed(mq[i], mk[j], qi == kj, flags);
    any |= a;
    all &= a;
  }
  any = __syncthreads_or(any);
  all = __syncthreads_and(all);
  if (threadIdx.x == 0)
    cls[((int64_t)b * nt + qt) * nt + kt] = any ? (all ? CLS_FULL : CLS_PARTIAL) : CLS_EMPTY;
}

// Forward lists: per (b, 128-row query tile) the non-empty 64-key tiles, class packed in the top
// bits (entry = kt | cls << 14).  Backward lists: per (b, 64-key tile) the non-empty 64-query
// tiles.  One thread per list.
__global__ void build_lists_kernel(const uint8_t* __restrict__ cls, int B, int nt, int16_t* __restrict__ fwd_list,
                                   int* __restrict__ fwd_cnt, int16_t* __restrict__ bwd_list,
                                   int* __restrict__ bwd_cnt) {
  const int nq2 = (nt + 1) / 2;
  const int tid = blockIdx.x * blockDim.x + threadIdx.x;
  const int nf = B * nq2, nb = B * nt;
  if (tid < nf) {
    const int b = tid / nq2, q2 = tid % nq2;
    int c = 0;
    for (int kt = 0; kt < nt; ++kt) {
      const int c0 = cls[((int64_t)b * nt + 2 * q2) * nt + kt];
      const int c1 = (2 * q2 + 1 < nt) ? cls[((int64_t)b * nt + 2 * q2 + 1) * nt + kt] : CLS_EMPTY;
      if (c0 == CLS_EMPTY && c1 == CLS_EMPTY) continue;
      // a half tile beyond T counts as partial (its rows are masked out of range anyway)
      const int cc = (c0 == CLS_FULL && (c1 == CLS_FULL || 2 * q2 + 1 >= nt)) ? CLS_FULL : CLS_PARTIAL;
      fwd_list[(int64_t)tid * nt + c] = (int16_t)(kt | (cc << 14));
      ++c;
    }
    fwd_cnt[tid] = c;
  } else if (tid < nf + nb) {
    const int t2 = tid - nf;
    const int b = t2 / nt, kt = t2 % nt;
    int c = 0;
    for (int qt = 0; qt < nt; ++qt) {
      const int cc = cls[((int64_t)b * nt + qt) * nt + kt];
      if (cc == CLS_EMPTY) continue;
      bwd_list[(int64_t)t2 * nt + c] = (int16_t)(qt | (cc << 14));
      ++c;
    }
    bwd_cnt[t2] = c;
  }
}

struct FwdParams {
  const bf16 *q, *k, *v;
  int64_t q_tok, k_tok, v_tok;     // token strides (elements)
  int64_t q_b, k_b, v_b;           // batch strides
  bf16* o; int64_t o_tok, o_b;
  float* lse;                      // [B, Hq, T]
  const int4* meta;
  const int16_t* list; const int* cnt;
  int T, Hq, group, nt, flags;
  float scale_log2;                // softmax scale * log2(e)
};

// ---- forward: CTA = 128 query rows (8 warps x 16) of one head; 64-key tiles ------------------
template <int D>
__global__ void __launch_bounds__(256) fwd_kernel(const FwdParams p) {
  constexpr int BM = 128, BN = 64, NT = 256;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  bf16* sQ = reinterpret_cast<bf16*>(smem_raw);
  bf16* sK = sQ + BM * D;
  bf16* sV = sK + 2 * BN * D;
  int4* sMq = reinterpret_cast<int4*>(sV + 2 * BN * D);
  int4* sMk = sMq + BM;

  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int hk = h / p.group;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nq2 = (p.nt + 1) / 2;
  const int lidx = b * nq2 + qt;
  const int n = p.cnt[lidx];
  const int16_t* list = p.list + (int64_t)lidx * p.nt;

  const bf16* gq = p.q + (int64_t)b * p.q_b + (int64_t)h * D;
  const bf16* gk = p.k + (int64_t)b * p.k_b + (int64_t)hk * D;
  const bf16* gv = p.v + (int64_t)b * p.v_b + (int64_t)hk * D;

  load_tile<D, BM, NT>(sQ, gq, p.q_tok, qt * BM, p.T);
  if (threadIdx.x < BM) sMq[threadIdx.x] = load_meta(p.meta, b, p.T, qt * BM + threadIdx.x);
  auto issue_kv = [&](int it) {
    const int kt = list[it] & 0x3fff;
    const int buf = it & 1;
    load_tile<D, BN, NT>(sK + buf * BN * D, gk, p.k_tok, kt * BN, p.T);
    load_tile<D, BN, NT>(sV + buf * BN * D, gv, p.v_tok, kt * BN, p.T);
    if (threadIdx.x < BN) sMk[buf * BN + threadIdx.x] = load_meta(p.meta, b, p.T, kt * BN + threadIdx.x);
  };
  if (n > 0) issue_kv(0);
  cp_async_commit();

  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_i[2] = {-INFINITY, -INFINITY}, l_i[2] = {0.f, 0.f};
  // Q fragments stay in registers for D <= 128; for D = 256 they are re-read from smem per tile
  // (ldmatrix is cheap) to keep the O accumulator and S tile within the register budget.
  constexpr bool QREG = D <= 128;
  uint32_t qf[QREG ? D / 16 : 1][4];
  const int wr = warp * 16;  // warp's first row in the tile
  const int r_lo = wr + (lane >> 2), r_hi = r_lo + 8;

  for (int it = 0; it < n; ++it) {
    if (it + 1 < n) issue_kv(it + 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (QREG && it == 0) {
#pragma unroll
      for (int kk = 0; kk < (QREG ? D / 16 : 0); ++kk) {
        const int row = wr + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int col = kk * 16 + (lane >> 4) * 8;
        ldsm_x4(qf[kk], sQ + swz<D>(row, col));
      }
    }
    const int buf = it & 1;
    const bf16* cK = sK + buf * BN * D;
    const bf16* cV = sV + buf * BN * D;
    const int4* cMk = sMk + buf * BN;
    const int entry = list[it];
    const int kt = entry & 0x3fff;
    const bool partial = (entry >> 14) != CLS_FULL;

    float s[BN / 8][4];
#pragma unroll
    for (int j = 0; j < BN / 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t qtmp[4];
      if constexpr (!QREG) {
        const int row = wr + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int col = kk * 16 + (lane >> 4) * 8;
        ldsm_x4(qtmp, sQ + swz<D>(row, col));
      }
      const uint32_t(&qa)[4] = QREG ? qf[QREG ? kk : 0] : qtmp;
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
    if (partial) {
      const int4 mlo = sMq[r_lo], mhi = sMq[r_hi];
      const int qlo = qt * BM + r_lo, qhi = qt * BM + r_hi;
#pragma unroll
      for (int j = 0; j < BN / 8; ++j) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int c = j * 8 + (lane & 3) * 2 + e;
          const int kj = kt * BN + c;
          const int4 mk = cMk[c];
          const bool kin = kj < p.T;
          if (!(kin && allowed(mlo, mk, qlo == kj, p.flags))) s[j][e] = -INFINITY;
          if (!(kin && allowed(mhi, mk, qhi == kj, p.flags))) s[j][2 + e] = -INFINITY;
        }
      }
    }
    // online softmax (rows r_lo -> elements 0,1 ; r_hi -> elements 2,3)
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
      // accumulator layout of S(16x8 tile j) == A-fragment layout of P(16x16 k-step j/2)
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
    // O += P V   (V is [key][d] row-major -> transposed ldmatrix gives the B fragment)
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
    __syncthreads();  // buffer `buf` is refilled by the next iteration's prefetch
  }

  // finalize
  float inv[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    float l = l_i[r];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    l_i[r] = l;
    inv[r] = l > 0.f ? 1.f / l : 0.f;
  }
  const int q0 = qt * BM;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = q0 + (r ? r_hi : r_lo);
    if (row >= p.T) continue;
    bf16* go = p.o + (int64_t)b * p.o_b + (int64_t)row * p.o_tok + (int64_t)h * D;
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      const int col = i * 8 + (lane & 3) * 2;
      *reinterpret_cast<__nv_bfloat162*>(go + col) =
          __floats2bfloat162_rn(o[i][2 * r] * inv[r], o[i][2 * r + 1] * inv[r]);
    }
    if ((lane & 3) == 0) {
      // natural-log LSE of the scaled scores
      const float lse = (m_i[r] == -INFINITY) ? -INFINITY
                                              : (m_i[r] * p.scale_log2 + log2f(l_i[r])) * 0.69314718055994530942f;
      p.lse[((int64_t)b * p.Hq + h) * p.T + row] = lse;
    }
  }
}

// ---- backward preprocessing: Dsum[b,h,t] = sum_d dO * O -------------------------------------
__global__ void bwd_dsum_kernel(const bf16* __restrict__ o, int64_t o_tok, int64_t o_b, const bf16* __restrict__ dout,
                                int64_t do_tok, int64_t do_b, float* __restrict__ dsum, int B, int T, int Hq, int D) {
  const int64_t gw = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (gw >= (int64_t)B * T * Hq) return;
  const int h = (int)(gw % Hq);
  const int t = (int)((gw / Hq) % T);
  const int b = (int)(gw / ((int64_t)Hq * T));
  const bf16* po = o + (int64_t)b * o_b + (int64_t)t * o_tok + (int64_t)h * D;
  const bf16* pd = dout + (int64_t)b * do_b + (int64_t)t * do_tok + (int64_t)h * D;
  float acc = 0.f;
  for (int c = lane * 8; c < D; c += 256) {
    float a[8], g[8];
    load8(po + c, a);
    load8(pd + c, g);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc += a[i] * g[i];
  }
  acc = warp_sum(acc);
  if (lane == 0) dsum[((int64_t)b * Hq + h) * T + t] = acc;
}

// Backward prologue of the tcgen05 path: Dsum[b, h, t] = sum_d O * dO for every query row, and
// the fp32 dQ / dK / dV accumulators of the same rows set to zero in the same pass (a row
// (b, t, h) zeroes dQ[b, t, h] and, when h is the first head of its GQA group, dK / dV[b, t, h /
// group]).  D / 8 lanes per row (8 bf16 each), and four rows per lane group loaded before the
// first reduction so each lane keeps 128 bytes in flight.
template <int D>
__global__ void __launch_bounds__(256) bwd_prep_kernel(const bf16* __restrict__ o, int64_t o_tok, int64_t o_b,
                                                       const bf16* __restrict__ dout, int64_t do_tok, int64_t do_b,
                                                       float* __restrict__ dsum, float* __restrict__ dq_acc,
                                                       float* __restrict__ dk_acc, float* __restrict__ dv_acc, int B,
                                                       int T, int Hq, int group) {
  constexpr int LPR = D / 8, RPW = 32 / LPR, U = 4;
  const int lane = threadIdx.x & 31, sub = lane / LPR, j = lane % LPR;
  const int64_t rows = (int64_t)B * T * Hq;
  const int Hkv = Hq / group;
  const int64_t step = (int64_t)gridDim.x * (blockDim.x >> 5) * RPW * U;
  for (int64_t base = ((int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * RPW * U; base < rows;
       base += step) {
    float a[U][8], g[U][8];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t row = base + u * RPW + sub;
      if (row < rows) {
        const int h = (int)(row % Hq);
        const int64_t bt = row / Hq;
        const int t = (int)(bt % T), b = (int)(bt / T);
        load8(o + (int64_t)b * o_b + (int64_t)t * o_tok + (int64_t)h * D + j * 8, a[u]);
        load8(dout + (int64_t)b * do_b + (int64_t)t * do_tok + (int64_t)h * D + j * 8, g[u]);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) a[u][i] = g[u][i] = 0.f;
      }
    }
    const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int u = 0; u < U; ++u) {
      float acc = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) acc += a[u][i] * g[u][i];
#pragma unroll
      for (int off = LPR / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
      const int64_t row = base + u * RPW + sub;
      if (row < rows) {
        const int h = (int)(row % Hq);
        const int64_t bt = row / Hq;
        const int t = (int)(bt % T), b = (int)(bt / T);
        if (j == 0) dsum[((int64_t)b * Hq + h) * T + t] = acc;
        if (dq_acc != nullptr) {   // the head_dim 256 tcgen05 backward writes dq without an accumulator
          float* q = dq_acc + row * D + j * 8;
          reinterpret_cast<float4*>(q)[0] = z;
          reinterpret_cast<float4*>(q)[1] = z;
        }
        if (dk_acc != nullptr && h % group == 0) {
          const int64_t kr = (bt * Hkv + h / group) * D + j * 8;
          reinterpret_cast<float4*>(dk_acc + kr)[0] = z;
          reinterpret_cast<float4*>(dk_acc + kr)[1] = z;
          reinterpret_cast<float4*>(dv_acc + kr)[0] = z;
          reinterpret_cast<float4*>(dv_acc + kr)[1] = z;
        }
      }
    }
  }
}

struct BwdParams {
  const bf16 *q, *k, *v, *dout;
  int64_t q_tok, k_tok, v_tok, do_tok;
  int64_t q_b, k_b, v_b, do_b;
  const float *lse, *dsum;          // [B, Hq, T]
  float* dq_acc;                    // [B, T, Hq, D] fp32 (zeroed)
  bf16 *dk, *dv;                    // dk [B,T,Hkv,D] contiguous; dv strided
  int64_t dk_tok, dk_b, dv_tok, dv_b;
  const int4* meta;
  const int16_t* list; const int* cnt;
  int T, Hq, group, nt, flags;
  float scale, scale_log2;
  int dcol0;                        // first head-dim column of dQ / dK / dV this launch produces
};

__device__ __forceinline__ void red_add_v2(float* addr, float a, float b) {
  asm volatile("red.global.add.v2.f32 [%0], {%1, %2};\n" ::"l"(addr), "f"(a), "f"(b) : "memory");
}

// ---- backward: CTA = 64 keys (4 warps x 16) of one KV head, looping over the GQA group's query
// heads and the non-empty 64-query tiles.  dK/dV accumulate in registers; dQ is reduced through
// shared memory and added to an fp32 global accumulator.  A launch produces the DH head-dim columns
// [dcol0, dcol0 + DH) of dQ / dK / dV (DH < D splits head_dim 256 over two launches that both
// recompute S and dP, keeping the dK / dV accumulators within the register file).
template <int D, int DH>
__global__ void __launch_bounds__(128) bwd_kernel(const BwdParams p) {
  constexpr int BN = 64, BM = 64, NT = 128;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  bf16* sK = reinterpret_cast<bf16*>(smem_raw);       // [BN][D]
  bf16* sV = sK + BN * D;                               // [BN][D]
  bf16* sQ = sV + BN * D;                               // [2][BM][D]
  bf16* sdO = sQ + 2 * BM * D;                          // [2][BM][D]
  bf16* sdS = sdO + 2 * BM * D;                         // [BM][BN] (dS, query-major, swizzled)
  int4* sMk = reinterpret_cast<int4*>(sdS + BM * BN);   // [BN]
  int4* sMq = sMk + BN;                                 // [2][BM]
  float* sL = reinterpret_cast<float*>(sMq + 2 * BM);   // [2][BM] lse
  float* sDs = sL + 2 * BM;                             // [2][BM] dsum

  const int kt = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int lidx = b * p.nt + kt;
  const int nq = p.cnt[lidx];
  const int16_t* list = p.list + (int64_t)lidx * p.nt;
  const int total = nq * p.group;

  load_tile<D, BN, NT>(sK, p.k + (int64_t)b * p.k_b + (int64_t)hk * D, p.k_tok, kt * BN, p.T);
  load_tile<D, BN, NT>(sV, p.v + (int64_t)b * p.v_b + (int64_t)hk * D, p.v_tok, kt * BN, p.T);
  if (threadIdx.x < BN) sMk[threadIdx.x] = load_meta(p.meta, b, p.T, kt * BN + threadIdx.x);

  auto issue_q = [&](int it) {
    const int g = it / nq, qi = it % nq;
    const int h = hk * p.group + g;
    const int qt = list[qi] & 0x3fff;
    const int buf = it & 1;
    load_tile<D, BM, NT>(sQ + buf * BM * D, p.q + (int64_t)b * p.q_b + (int64_t)h * D, p.q_tok, qt * BM, p.T);
    load_tile<D, BM, NT>(sdO + buf * BM * D, p.dout + (int64_t)b * p.do_b + (int64_t)h * D, p.do_tok, qt * BM, p.T);
    if (threadIdx.x < BM) {
      const int row = qt * BM + threadIdx.x;
      sMq[buf * BM + threadIdx.x] = load_meta(p.meta, b, p.T, row);
      const int64_t li = ((int64_t)b * p.Hq + h) * p.T + row;
      sL[buf * BM + threadIdx.x] = row < p.T ? p.lse[li] : 0.f;
      sDs[buf * BM + threadIdx.x] = row < p.T ? p.dsum[li] : 0.f;
    }
  };
  if (total > 0) issue_q(0);
  cp_async_commit();

  const int dc0 = p.dcol0;
  float dk[DH / 8][4], dv[DH / 8][4];
#pragma unroll
  for (int i = 0; i < DH / 8; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) dk[i][e] = dv[i][e] = 0.f;

  const int wr = warp * 16;                         // warp's first key row
  const int k_lo = wr + (lane >> 2), k_hi = k_lo + 8;

  for (int it = 0; it < total; ++it) {
    if (it + 1 < total) issue_q(it + 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const int buf = it & 1;
    const int g = it / nq, qi = it % nq;
    const int h = hk * p.group + g;
    const int entry = list[qi];
    const int qt = entry & 0x3fff;
    const bool partial = (entry >> 14) != CLS_FULL;
    const bf16* cQ = sQ + buf * BM * D;
    const bf16* cdO = sdO + buf * BM * D;
    const int4* cMq = sMq + buf * BM;
    const float* cL = sL + buf * BM;
    const float* cDs = sDs + buf * BM;

    // S^T = K Q^T  (warp rows = 16 keys, cols = 64 queries)
    float st[BM / 8][4];
#pragma unroll
    for (int j = 0; j < BM / 8; ++j) st[j][0] = st[j][1] = st[j][2] = st[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t af[4];
      {
        const int row = wr + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int col = kk * 16 + (lane >> 4) * 8;
        ldsm_x4(af, sK + swz<D>(row, col));
      }
#pragma unroll
      for (int jp = 0; jp < BM / 16; ++jp) {
        uint32_t bfr[4];
        const int row = jp * 16 + (lane & 7) + (lane >> 4) * 8;
        const int col = kk * 16 + ((lane >> 3) & 1) * 8;
        ldsm_x4(bfr, cQ + swz<D>(row, col));
        mma16816(st[2 * jp], af, bfr[0], bfr[1]);
        mma16816(st[2 * jp + 1], af, bfr[2], bfr[3]);
      }
    }
    // P^T = exp(S^T * scale - lse[q]) with the mask
    const int4 mklo = sMk[k_lo], mkhi = sMk[k_hi];
    const int kjlo = kt * BN + k_lo, kjhi = kt * BN + k_hi;
#pragma unroll
    for (int j = 0; j < BM / 8; ++j) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int c = j * 8 + (lane & 3) * 2 + e;
        const int qrow = qt * BM + c;
        const float L = cL[c] * 1.44269504088896340736f;
        bool alo = qrow < p.T && kjlo < p.T, ahi = qrow < p.T && kjhi < p.T;
        if (partial) {
          const int4 mq = cMq[c];
          alo = alo && allowed(mq, mklo, qrow == kjlo, p.flags);
          ahi = ahi && allowed(mq, mkhi, qrow == kjhi, p.flags);
        }
        st[j][e] = alo ? exp2f(st[j][e] * p.scale_log2 - L) : 0.f;
        st[j][2 + e] = ahi ? exp2f(st[j][2 + e] * p.scale_log2 - L) : 0.f;
      }
    }
    // dV += P^T dO
    {
      uint32_t pf[BM / 16][4];
#pragma unroll
      for (int j = 0; j < BM / 8; ++j) {
        pf[j >> 1][(j & 1) * 2 + 0] = pack_bf16(st[j][0], st[j][1]);
        pf[j >> 1][(j & 1) * 2 + 1] = pack_bf16(st[j][2], st[j][3]);
      }
#pragma unroll
      for (int kk = 0; kk < BM / 16; ++kk) {
#pragma unroll
        for (int dp = 0; dp < DH / 16; ++dp) {
          uint32_t bfr[4];
          const int row = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
          const int col = dc0 + dp * 16 + (lane >> 4) * 8;
          ldsm_x4_t(bfr, cdO + swz<D>(row, col));
          mma16816(dv[2 * dp], pf[kk], bfr[0], bfr[1]);
          mma16816(dv[2 * dp + 1], pf[kk], bfr[2], bfr[3]);
        }
      }
    }
    // dP^T = V dO^T
    float dpt[BM / 8][4];
#pragma unroll
    for (int j = 0; j < BM / 8; ++j) dpt[j][0] = dpt[j][1] = dpt[j][2] = dpt[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t af[4];
      {
        const int row = wr + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int col = kk * 16 + (lane >> 4) * 8;
        ldsm_x4(af, sV + swz<D>(row, col));
      }
#pragma unroll
      for (int jp = 0; jp < BM / 16; ++jp) {
        uint32_t bfr[4];
        const int row = jp * 16 + (lane & 7) + (lane >> 4) * 8;
        const int col = kk * 16 + ((lane >> 3) & 1) * 8;
        ldsm_x4(bfr, cdO + swz<D>(row, col));
        mma16816(dpt[2 * jp], af, bfr[0], bfr[1]);
        mma16816(dpt[2 * jp + 1], af, bfr[2], bfr[3]);
      }
    }
    // dS^T = P^T * (dP^T - Dsum[q]);  (the softmax scale is applied to dK/dQ at the end)
    uint32_t dsf[BM / 16][4];
#pragma unroll
    for (int j = 0; j < BM / 8; ++j) {
      float v4[4];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int c = j * 8 + (lane & 3) * 2 + e;
        const float ds = cDs[c];
        v4[e] = st[j][e] * (dpt[j][e] - ds);
        v4[2 + e] = st[j][2 + e] * (dpt[j][2 + e] - ds);
      }
      dsf[j >> 1][(j & 1) * 2 + 0] = pack_bf16(v4[0], v4[1]);
      dsf[j >> 1][(j & 1) * 2 + 1] = pack_bf16(v4[2], v4[3]);
      // stash dS (query-major) for the dQ product: element (key k, query c) -> sdS[c][k]
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int c = j * 8 + (lane & 3) * 2 + e;
        sdS[swz<BN>(c, k_lo)] = __float2bfloat16(v4[e]);
        sdS[swz<BN>(c, k_hi)] = __float2bfloat16(v4[2 + e]);
      }
    }
    // dK += dS^T Q
#pragma unroll
    for (int kk = 0; kk < BM / 16; ++kk) {
#pragma unroll
      for (int dp = 0; dp < DH / 16; ++dp) {
        uint32_t bfr[4];
        const int row = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int col = dc0 + dp * 16 + (lane >> 4) * 8;
        ldsm_x4_t(bfr, cQ + swz<D>(row, col));
        mma16816(dk[2 * dp], dsf[kk], bfr[0], bfr[1]);
        mma16816(dk[2 * dp + 1], dsf[kk], bfr[2], bfr[3]);
      }
    }
    __syncthreads();  // sdS complete
    // dQ[64 q x D] = dS[64 q x 64 k] K[64 k x D]; warp w owns queries 16w..16w+15
    {
      uint32_t af[BN / 16][4];
#pragma unroll
      for (int kk = 0; kk < BN / 16; ++kk) {
        const int row = wr + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int col = kk * 16 + (lane >> 4) * 8;
        ldsm_x4(af[kk], sdS + swz<BN>(row, col));
      }
      const int qlo = qt * BM + wr + (lane >> 2), qhi = qlo + 8;
      float* dqb = p.dq_acc + (int64_t)b * p.T * p.Hq * D + (int64_t)h * D;
#pragma unroll
      for (int dp = 0; dp < DH / 16; ++dp) {
        float acc0[4] = {0.f, 0.f, 0.f, 0.f}, acc1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          uint32_t bfr[4];
          const int row = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
          const int col = dc0 + dp * 16 + (lane >> 4) * 8;
          ldsm_x4_t(bfr, sK + swz<D>(row, col));
          mma16816(acc0, af[kk], bfr[0], bfr[1]);
          mma16816(acc1, af[kk], bfr[2], bfr[3]);
        }
        const int c0 = dc0 + dp * 16 + (lane & 3) * 2;
        if (qlo < p.T) {
          red_add_v2(dqb + (int64_t)qlo * p.Hq * D + c0, acc0[0] * p.scale, acc0[1] * p.scale);
          red_add_v2(dqb + (int64_t)qlo * p.Hq * D + c0 + 8, acc1[0] * p.scale, acc1[1] * p.scale);
        }
        if (qhi < p.T) {
          red_add_v2(dqb + (int64_t)qhi * p.Hq * D + c0, acc0[2] * p.scale, acc0[3] * p.scale);
          red_add_v2(dqb + (int64_t)qhi * p.Hq * D + c0 + 8, acc1[2] * p.scale, acc1[3] * p.scale);
        }
      }
    }
    __syncthreads();  // sdS / Q buffers are reused next iteration
  }
  // write dK (scaled) and dV
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = kt * BN + (r ? k_hi : k_lo);
    if (row >= p.T) continue;
    bf16* gdk = p.dk + (int64_t)b * p.dk_b + (int64_t)row * p.dk_tok + (int64_t)hk * D;
    bf16* gdv = p.dv + (int64_t)b * p.dv_b + (int64_t)row * p.dv_tok + (int64_t)hk * D;
#pragma unroll
    for (int i = 0; i < DH / 8; ++i) {
      const int col = dc0 + i * 8 + (lane & 3) * 2;
      *reinterpret_cast<__nv_bfloat162*>(gdk + col) =
          __floats2bfloat162_rn(dk[i][2 * r] * p.scale, dk[i][2 * r + 1] * p.scale);
      *reinterpret_cast<__nv_bfloat162*>(gdv + col) = __floats2bfloat162_rn(dv[i][2 * r], dv[i][2 * r + 1]);
    }
  }
}

__global__ void dq_convert_kernel(const float* __restrict__ acc, bf16* __restrict__ dq, int64_t dq_tok, int64_t dq_b,
                                  int B, int T, int Hq, int D) {
  const int64_t n8 = (int64_t)B * T * Hq * D / 8;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = i * 8;
    const int c = (int)(e % ((int64_t)Hq * D));
    const int t = (int)((e / ((int64_t)Hq * D)) % T);
    const int b = (int)(e / ((int64_t)Hq * D * T));
    const float4 a0 = *reinterpret_cast<const float4*>(acc + e);
    const float4 a1 = *reinterpret_cast<const float4*>(acc + e + 4);
    float f[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    store8(dq + (int64_t)b * dq_b + (int64_t)t * dq_tok + c, f);
  }
}

template <int D>
size_t fwd_smem() { return (size_t)(128 * D + 4 * 64 * D) * 2 + (128 + 2 * 64) * 16; }
template <int D>
size_t bwd_smem() { return (size_t)(2 * 64 * D + 4 * 64 * D + 64 * 64) * 2 + (64 + 2 * 64) * 16 + 4 * 64 * 4; }

}  // namespace attn

// ---------------------------------------------------------------------------------------------
void bd_attn_plan(const int4* meta, int B, int T, int flags, uint8_t* cls, int16_t* fwd_list, int* fwd_cnt,
                  int16_t* bwd_list, int* bwd_cnt, cudaStream_t s) {
  const int nt = ceil_div(T, attn::TILE);
  attn::classify_kernel<<<dim3(nt, nt, B), 256, 0, s>>>(meta, T, flags, cls);
  const int nq2 = (nt + 1) / 2;
  const int threads = B * nq2 + B * nt;
  attn::build_lists_kernel<<<ceil_div(threads, 128), 128, 0, s>>>(cls, B, nt, fwd_list, fwd_cnt, bwd_list, bwd_cnt);
}

template <int D>
static void launch_fwd(const attn::FwdParams& p, int B, cudaStream_t s) {
  static bool init = false;
  const size_t sm = attn::fwd_smem<D>();
  if (!init) {
    cudaFuncSetAttribute(attn::fwd_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    init = true;
  }
  dim3 grid((p.nt + 1) / 2, p.Hq, B);
  attn::fwd_kernel<D><<<grid, 256, sm, s>>>(p);
}

template <int D>
static void launch_bwd(attn::BwdParams p, int B, int Hkv, cudaStream_t s) {
  constexpr int DH = D > 128 ? 128 : D;
  static bool init = false;
  const size_t sm = attn::bwd_smem<D>();
  if (!init) {
    cudaFuncSetAttribute(attn::bwd_kernel<D, DH>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    init = true;
  }
  dim3 grid(p.nt, Hkv, B);
  for (int c0 = 0; c0 < D; c0 += DH) {
    p.dcol0 = c0;
    attn::bwd_kernel<D, DH><<<grid, 128, sm, s>>>(p);
  }
}

int bd_attn_fwd(const AttnTensors& t, const int4* meta, const int16_t* fwd_list, const int* fwd_cnt, int flags,
                float scale, cudaStream_t s) {
  attn::FwdParams p;
  p.q = t.q; p.k = t.k; p.v = t.v;
  p.q_tok = t.q_tok; p.k_tok = t.k_tok; p.v_tok = t.v_tok;
  p.q_b = t.q_b; p.k_b = t.k_b; p.v_b = t.v_b;
  p.o = t.o; p.o_tok = t.o_tok; p.o_b = t.o_b;
  p.lse = t.lse; p.meta = meta; p.list = fwd_list; p.cnt = fwd_cnt;
  p.T = t.T; p.Hq = t.Hq; p.group = t.Hq / t.Hkv; p.nt = ceil_div(t.T, attn::TILE); p.flags = flags;
  p.scale_log2 = scale * 1.44269504088896340736f;
  switch (t.D) {
    case 64: launch_fwd<64>(p, t.B, s); break;
    case 128: launch_fwd<128>(p, t.B, s); break;
    case 256: launch_fwd<256>(p, t.B, s); break;
    default: return -1;
  }
  return 0;
}

void bd_attn_bwd_prep(const AttnTensors& t, const bf16* dout, int64_t do_tok, int64_t do_b, float* dsum, float* dq_acc,
                      float* dk_acc, float* dv_acc, int sm_count, cudaStream_t s) {
  const int64_t rows = (int64_t)t.B * t.T * t.Hq;
  const bool vec = (t.D == 64 || t.D == 128 || t.D == 256) && t.o_tok % 8 == 0 && t.o_b % 8 == 0 &&
                   do_tok % 8 == 0 && do_b % 8 == 0 && (reinterpret_cast<uintptr_t>(t.o) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(dout) & 15) == 0;
  if (vec) {
    const int64_t per_block = 8 * (256 / t.D) * 4;   // rows a block covers per step
    int64_t blocks = (rows + per_block - 1) / per_block;
    blocks = blocks > (int64_t)sm_count * 8 ? (int64_t)sm_count * 8 : blocks;
    const int group = t.Hq / t.Hkv;
#define TRIDA_PREP(DD)                                                                                        \
  attn::bwd_prep_kernel<DD><<<(int)blocks, 256, 0, s>>>(t.o, t.o_tok, t.o_b, dout, do_tok, do_b, dsum, dq_acc, \
                                                        dk_acc, dv_acc, t.B, t.T, t.Hq, group)
    if (t.D == 64) TRIDA_PREP(64); else if (t.D == 128) TRIDA_PREP(128); else TRIDA_PREP(256);
#undef TRIDA_PREP
    return;
  }
  attn::bwd_dsum_kernel<<<ceil_div(rows, 8), 256, 0, s>>>(t.o, t.o_tok, t.o_b, dout, do_tok, do_b, dsum, t.B, t.T,
                                                           t.Hq, t.D);
  if (dq_acc != nullptr) cudaMemsetAsync(dq_acc, 0, sizeof(float) * rows * t.D, s);
  if (dk_acc != nullptr) {
    cudaMemsetAsync(dk_acc, 0, sizeof(float) * (int64_t)t.B * t.T * t.Hkv * t.D, s);
    cudaMemsetAsync(dv_acc, 0, sizeof(float) * (int64_t)t.B * t.T * t.Hkv * t.D, s);
  }
}

void bd_attn_dq_convert(const float* dq_acc, bf16* dq, int64_t dq_tok, int64_t dq_b, int B, int T, int Hq, int D,
                        int sm_count, cudaStream_t s) {
  const int64_t n8 = (int64_t)B * T * Hq * D / 8;
  int blocks = ceil_div(n8, 256);
  blocks = blocks > sm_count * 16 ? sm_count * 16 : blocks;
  attn::dq_convert_kernel<<<blocks, 256, 0, s>>>(dq_acc, dq, dq_tok, dq_b, B, T, Hq, D);
}

int bd_attn_bwd(const AttnTensors& t, const bf16* dout, int64_t do_tok, int64_t do_b, float* dsum, float* dq_acc,
                bf16* dq, int64_t dq_tok, int64_t dq_b, bf16* dk, int64_t dk_tok, int64_t dk_b, bf16* dv,
                int64_t dv_tok, int64_t dv_b, const int4* meta, const int16_t* bwd_list, const int* bwd_cnt,
                int flags, float scale, int sm_count, cudaStream_t s) {
  const int64_t rows = (int64_t)t.B * t.T * t.Hq;
  attn::bwd_dsum_kernel<<<ceil_div(rows, 8), 256, 0, s>>>(t.o, t.o_tok, t.o_b, dout, do_tok, do_b, dsum, t.B, t.T,
                                                           t.Hq, t.D);
  cudaMemsetAsync(dq_acc, 0, sizeof(float) * rows * t.D, s);
  attn::BwdParams p;
  p.q = t.q; p.k = t.k; p.v = t.v; p.dout = dout;
  p.q_tok = t.q_tok; p.k_tok = t.k_tok; p.v_tok = t.v_tok; p.do_tok = do_tok;
  p.q_b = t.q_b; p.k_b = t.k_b; p.v_b = t.v_b; p.do_b = do_b;
  p.lse = t.lse; p.dsum = dsum; p.dq_acc = dq_acc;
  p.dk = dk; p.dv = dv; p.dk_tok = dk_tok; p.dk_b = dk_b; p.dv_tok = dv_tok; p.dv_b = dv_b;
  p.meta = meta; p.list = bwd_list; p.cnt = bwd_cnt;
  p.T = t.T; p.Hq = t.Hq; p.group = t.Hq / t.Hkv; p.nt = ceil_div(t.T, attn::TILE); p.flags = flags;
  p.scale = scale; p.scale_log2 = scale * 1.44269504088896340736f;
  switch (t.D) {
    case 64: launch_bwd<64>(p, t.B, t.Hkv, s); break;
    case 128: launch_bwd<128>(p, t.B, t.Hkv, s); break;
    case 256: launch_bwd<256>(p, t.B, t.Hkv, s); break;
    default: return -1;
  }
  const int64_t n8 = rows * t.D / 8;
  int blocks = ceil_div(n8, 256);
  blocks = blocks > sm_count * 16 ? sm_count * 16 : blocks;
  attn::dq_convert_kernel<<<blocks, 256, 0, s>>>(dq_acc, dq, dq_tok, dq_b, t.B, t.T, t.Hq, t.D);
  return 0;
}

}  // namespace trida
