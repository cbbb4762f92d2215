// Block-diffusion attention for head_dim 256 (the Qwen3.5-style full-attention layers) on the
// 5th-generation tensor cores: forward, and a backward split into a dK / dV kernel and a dQ kernel.
//
// Why a separate design from the head_dim 64 / 128 kernels: a [128 rows][256] bf16 tile is 64 KB,
// so two such tiles resident plus a double-buffered pair no longer fit in 227 KB of shared memory,
// and a 128-row fp32 accumulator of 256 columns takes half of the 512 TMEM columns.  So:
//   * tiles move in 64-column sub-tiles ([128 rows][64 bf16], 16 KB, 128-byte swizzled, one TMA box)
//     through small rings, and each contraction over d walks its sub-tiles in the order they arrive;
//   * forward: TMEM = S0 | S1 | O (128 + 128 + 256 columns); Q stays in shared memory (the A
//     operand of S = Q K^T), P is written over S in TMEM and is the A operand of O += P V;
//   * backward dK / dV: one CTA per (128-key tile, query head, half of d).  TMEM = S^T | dP^T |
//     dV_half | dK_half; S^T and dP^T contract over all of d, then P^T and dS^T are written over
//     them in TMEM as bf16 and are the A operands of dV_half += P^T dO[:, half] and
//     dK_half += dS^T Q[:, half].  The two halves recompute S^T / dP^T (1.5x the MMA work of those
//     two products) so that both accumulators stay in TMEM;
//   * backward dQ: one CTA per (128-query tile, query head) over its key tiles (the forward's tile
//     list and row masks): S = Q K^T and dP = dO V^T from resident Q / dO, dS written over S in
//     TMEM, dQ += dS K into 256 TMEM columns, stored once as bf16 (no fp32 dQ accumulator).
// Warp roles as in the other attention kernels: warps 0-7 elementwise (thread (g, r) owns TMEM lane
// r and one 64-column half of the 128-column S tile), warp 8 issues MMAs (one thread), warp 9
// issues TMA loads (one thread).  Every mbarrier wait is bounded and records an error code.
#include <cudaTypedefs.h>

#include "common.cuh"
#include "ops.h"
#include "sm100_common.cuh"
#include "bd_attention_sm100.cuh"

#include <climits>

namespace trida {
namespace attn256 {

using namespace sm100;
using attn100::CLS_FULL;
using attn100::fast_exp2;
using attn100::named_sync;
using attn100::RESCALE_THRESHOLD;

constexpr int BM = 128;
constexpr int SUB = 128 * 128;      // bytes of one [128 rows][64 bf16] sub-tile
constexpr int NTH = 320;            // 8 elementwise warps + MMA warp + TMA warp
constexpr int RING = 5;             // forward: K / V ring of 5 units (a unit = 2 sub-tiles = 128 of d)

__device__ __forceinline__ void named_bar_sync_256() { attn100::named_bar_sync(1, 256); }

struct FwdParams {
  float* lse;            // [B, Hq, T]
  const int4* meta;
  const int16_t* list;   // [B, nq, nk] entries kt | cls << 14
  const int* cnt;        // [B, nq]
  const uint4* tmask;    // [B, nq, nk, 128] row masks of PARTIAL tiles
  int* err;
  int T, Hq, group, nk, flags;
  float scale_log2;
};

// Forward shared memory: Q (4 sub-tiles, later the O staging tile), the K / V unit ring, the
// half-row max / sum exchange and the barriers.
struct FwdSmem {
  static constexpr int Q = 0;
  static constexpr int R0 = Q + 4 * SUB;
  static constexpr int XCH = R0 + RING * 2 * SUB;
  static constexpr int BAR = XCH + 2 * BM * 4;
  static constexpr int TOTAL = BAR + 256;
};
static_assert(FwdSmem::TOTAL + 1024 <= 232448, "forward shared memory");

// Forward.  The producer streams K_0, then (K_i, V_{i-1}) for i >= 1, then V_{n-1}, as units of 128
// d-columns (two sub-tiles); the MMA warp consumes them in the same order: S_0, then S_i and
// PV_{i-1} alternately, then PV_{n-1}, so the softmax of tile i-1 overlaps S_i.
__global__ void __launch_bounds__(NTH, 1)
    fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
               const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO, const FwdParams p) {
  using S = FwdSmem;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::BAR);
  uint64_t* q_full = bars + 0;
  uint64_t* u_full = bars + 1;       // [RING]
  uint64_t* u_empty = bars + 6;      // [RING]
  uint64_t* s_full = bars + 11;      // [2]
  // [2]: P_i written completes p_full[i & 1] (S_{i+1} is issued before PV_i, so a softmax warp can
  // finish tile i+1 while another is still on tile i; one barrier per parity keeps their arrivals apart)
  uint64_t* p_full = bars + 13;
  uint64_t* pv_done = bars + 15;     // [2]
  uint64_t* drain = bars + 17;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 18);

  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int hk = h / p.group;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nq = gridDim.x;
  const int lidx = b * nq + qt;
  const int n = p.cnt[lidx];
  const int16_t* list = p.list + (int64_t)lidx * p.nk;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int j = 0; j < RING; ++j) {
      mbar_init(&u_full[j], 1);
      mbar_init(&u_empty[j], 1);
    }
    mbar_init(&s_full[0], 1);
    mbar_init(&s_full[1], 1);
    mbar_init(&p_full[0], 2 * BM);
    mbar_init(&p_full[1], 2 * BM);
    mbar_init(&pv_done[0], 1);
    mbar_init(&pv_done[1], 1);
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS[2] = {tmem, tmem + 128};
  const uint32_t tO = tmem + 256;

  if (warp == 9) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      mbar_expect_tx(q_full, 4 * SUB);
#pragma unroll
      for (int c = 0; c < 4; ++c) tma_load_4d(smem + S::Q + c * SUB, &tmQ, q_full, c * 64, h, qt * BM, b);
      int u = 0;
      auto load_tile = [&](const CUtensorMap* map, int kt) {
        for (int hf = 0; hf < 2; ++hf, ++u) {
          const int slot = u % RING;
          if (u >= RING && !mbar_wait(&u_empty[slot], (u / RING - 1) & 1, p.err, 1)) return false;
          mbar_expect_tx(&u_full[slot], 2 * SUB);
          for (int c = 0; c < 2; ++c)
            tma_load_4d(smem + S::R0 + (slot * 2 + c) * SUB, map, &u_full[slot], (hf * 2 + c) * 64, hk, kt * BM, b);
        }
        return true;
      };
      bool ok = n == 0 || load_tile(&tmK, list[0] & 0x3fff);
      for (int i = 1; ok && i < n; ++i)
        ok = load_tile(&tmK, list[i] & 0x3fff) && load_tile(&tmV, list[i - 1] & 0x3fff);
      if (ok && n > 0) ok = load_tile(&tmV, list[n - 1] & 0x3fff);
      // the last units must have landed before the CTA can retire
      for (int v = (u > RING ? u - RING : 0); ok && v < u; ++v) mbar_wait(&u_full[v % RING], (v / RING) & 1, p.err, 2);
    }
  } else if (warp == 8) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16_f32(BM, 128, 0, 0);
      constexpr uint32_t idPV = idesc_bf16_f32(BM, 128, 0, 1);
      const uint32_t sQ = smem_addr(smem + S::Q), sR = smem_addr(smem + S::R0);
      bool ok = mbar_wait(q_full, 0, p.err, 3);
      int u = 0;
      auto issue_s = [&](int i) {
        const int s = i & 1;
        // S_i goes over P_{i-2} in TMEM: PV_{i-2} must have read it
        if (i >= 2 && !mbar_wait(&pv_done[s], ((i - 2) >> 1) & 1, p.err, 11)) return false;
        for (int hf = 0; hf < 2; ++hf, ++u) {
          const int slot = u % RING;
          if (!mbar_wait(&u_full[slot], (u / RING) & 1, p.err, 4)) return false;
          tc_fence_after();
          const uint32_t base = sR + slot * 2 * SUB;
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const int kg = hf * 8 + k;   // 16-column step over d
            umma_f16(tS[s], desc_sw128(sQ + (kg >> 2) * SUB + (kg & 3) * 32, 16, 1024),
                     desc_sw128(base + (k >> 2) * SUB + (k & 3) * 32, 16, 1024), idS, kg > 0 ? 1u : 0u);
          }
          umma_commit(&u_empty[slot]);
        }
        umma_commit(&s_full[s]);
        return true;
      };
      auto issue_pv = [&](int j) {
        const uint32_t pcol = tS[j & 1];
        for (int hf = 0; hf < 2; ++hf, ++u) {
          const int slot = u % RING;
          if (!mbar_wait(&u_full[slot], (u / RING) & 1, p.err, 13)) return false;
          tc_fence_after();
          const uint32_t base = sR + slot * 2 * SUB;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            // keys [16 kk, 16 kk + 16): P written by half kk / 4 at column 64 (kk / 4) + 8 (kk % 4)
            umma_f16_ts(tO + hf * 128, pcol + (kk >> 2) * 64 + (kk & 3) * 8, desc_sw128(base + kk * 2048, SUB, 1024),
                        idPV, (j > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&u_empty[slot]);
        }
        umma_commit(&pv_done[j & 1]);
        return true;
      };
      if (ok && n > 0) ok = issue_s(0);
      for (int i = 1; ok && i < n; ++i) {
        if (!(ok = issue_s(i))) break;
        if (!(ok = mbar_wait(&p_full[(i - 1) & 1], ((i - 1) >> 1) & 1, p.err, 5))) break;
        tc_fence_after();
        ok = issue_pv(i - 1);
      }
      if (ok && n > 0 && mbar_wait(&p_full[(n - 1) & 1], ((n - 1) >> 1) & 1, p.err, 6)) {
        tc_fence_after();
        issue_pv(n - 1);
      }
      umma_commit(drain);
      mbar_wait(drain, 0, p.err, 7);
    }
  } else {
    // ---------------- softmax / correction / epilogue (warps 0-7) ----------------
    const int half = warp >> 2;             // columns [64 half, 64 half + 64) of the S tile
    const int r = (warp & 3) * 32 + lane;   // query row within the tile == TMEM lane
    const int row = qt * BM + r;
    const int bar_id = 1 + (warp & 3);      // named barrier of warps (w, w + 4)
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    float* xch = reinterpret_cast<float*>(smem + S::XCH);
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int i = 0; i < n; ++i) {
      const int s = i & 1;
      const int entry = list[i];
      const int kt = entry & 0x3fff;
      const bool partial = (entry >> 14) != CLS_FULL;
      uint32_t bits[2] = {0xffffffffu, 0xffffffffu};
      if (partial) {
        const uint4 w = p.tmask[(((int64_t)b * nq + qt) * p.nk + kt) * BM + r];
        bits[0] = half ? w.z : w.x;
        bits[1] = half ? w.w : w.y;
      }
      if (ok) ok = mbar_wait(&s_full[s], (i >> 1) & 1, p.err, 8);
      float sv[64];
      float mx = -INFINITY;
      if (ok) {
        tc_fence_after();
        uint32_t t[2][32];
        tmem_ld32(tS[s] + lane_off + half * 64, t[0]);
        tmem_ld32(tS[s] + lane_off + half * 64 + 32, t[1]);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int j = 0; j < 32; ++j) sv[c * 32 + j] = __uint_as_float(t[c][j]);
        if (partial) {
#pragma unroll
          for (int c = 0; c < 64; ++c)
            if (!((bits[c >> 5] >> (c & 31)) & 1u)) sv[c] = -INFINITY;
        }
        float mxp[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) mxp[u] = sv[u];
#pragma unroll
        for (int c = 8; c < 64; ++c) mxp[c & 7] = fmaxf(mxp[c & 7], sv[c]);
        mx = fmaxf(fmaxf(fmaxf(mxp[0], mxp[1]), fmaxf(mxp[2], mxp[3])),
                   fmaxf(fmaxf(mxp[4], mxp[5]), fmaxf(mxp[6], mxp[7])));
      }
      // row max over both halves (the pair meets the barrier even after a timed-out wait)
      xch[half * BM + r] = mx;
      named_sync(bar_id, 64);
      mx = fmaxf(mx, xch[(1 - half) * BM + r]);
      named_sync(bar_id, 64);
      const float mx_s = mx * p.scale_log2;
      const bool grow = mx_s > m_run + RESCALE_THRESHOLD || (m_run == -INFINITY && mx_s > -INFINITY);
      // O may be rescaled only after PV_{i-1} has completed.  TMEM loads / stores are
      // warp-collective, so when any row of the warp rescales, every lane waits for PV_{i-1},
      // loads and stores its O columns (alpha = 1 for rows that keep their max)
      const bool resc = grow && i > 0 && m_run != -INFINITY;
      if (__any_sync(0xffffffffu, resc && ok)) {
        if (ok) ok = mbar_wait(&pv_done[(i - 1) & 1], ((i - 1) >> 1) & 1, p.err, 9);
        tc_fence_after();
        const float alpha = (resc && ok) ? exp2f(m_run - mx_s) : 1.f;
        l_run *= alpha;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {            // this half's columns of the O row
          uint32_t t[32];
          const uint32_t col = tO + lane_off + half * 128 + c * 32;
          tmem_ld32(col, t);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) t[j] = __float_as_uint(__uint_as_float(t[j]) * alpha);
          tmem_st32(col, t);
        }
        tmem_wait_st();
      }
      if (grow) m_run = mx_s;
      if (ok) {
        // P_i (bf16 pairs) over this half's own S_i columns: 32 columns from column 64 half
        const float m_use = (m_run == -INFINITY) ? 0.f : m_run;
        float rsp[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        uint32_t pw[32];
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8) {
          float pv[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            pv[j] = fast_exp2(sv[c8 * 8 + j] * p.scale_log2 - m_use);
            rsp[j] += pv[j];
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const __nv_bfloat162 t2 = __floats2bfloat162_rn(pv[2 * j], pv[2 * j + 1]);
            pw[c8 * 4 + j] = *reinterpret_cast<const uint32_t*>(&t2);
          }
        }
        tmem_st32(tS[s] + lane_off + half * 64, pw);
        tmem_wait_st();
        l_run += ((rsp[0] + rsp[1]) + (rsp[2] + rsp[3])) + ((rsp[4] + rsp[5]) + (rsp[6] + rsp[7]));
      }
      tc_fence_before();
      mbar_arrive(&p_full[i & 1]);
    }
    if (ok && n > 0) ok = mbar_wait(&pv_done[(n - 1) & 1], ((n - 1) >> 1) & 1, p.err, 10);
    xch[half * BM + r] = l_run;
    named_sync(bar_id, 64);
    const float l_tot = l_run + xch[(1 - half) * BM + r];
    // epilogue: O / l staged as bf16 in the idle Q tile (every S MMA has completed), then written
    // by TMA as whole 128-row sub-tiles (rows past T clipped)
    unsigned char* sO = smem + S::Q;
    const bool store = ok && n > 0;
    if (store) {
      tc_fence_after();
      const float inv = l_tot > 0.f ? 1.f / l_tot : 0.f;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t t[32];
        tmem_ld32(tO + lane_off + half * 128 + c * 32, t);
        tmem_wait_ld();
#pragma unroll
        for (int j8 = 0; j8 < 4; ++j8) {
          float f[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) f[j] = __uint_as_float(t[j8 * 8 + j]) * inv;
          const int col = half * 128 + c * 32 + j8 * 8;
          store8(reinterpret_cast<bf16*>(sO + (col >> 6) * SUB + sw128_offset(r, col & 63)), f);
        }
      }
      if (half == 0 && row < p.T)
        p.lse[((int64_t)b * p.Hq + h) * p.T + row] =
            (m_run == -INFINITY) ? -INFINITY : (m_run + log2f(l_tot)) * 0.69314718055994530942f;
      fence_async_smem();
    }
    named_sync(5, 256);
    if (threadIdx.x == 0 && store) {
#pragma unroll
      for (int c = 0; c < 4; ++c) attn100::tma_store_4d(&tmO, sO + c * SUB, c * 64, h, qt * BM, b);
      attn100::bulk_commit();
      attn100::bulk_wait_all();
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

// =================================================================================================
// Backward, dK / dV.  CTA = (128-key tile kt, query head h, half hf of d).  Per non-empty query tile
// j of the key tile (thread (g, r) of warps 0-7 owns key row r == TMEM lane r and query columns
// [64 g, 64 g + 64)):
//   S^T  = K Q_j^T    -> TMEM [0,128)     A = K (resident), B = Q_j: the other half's two sub-tiles
//                                          (transient ring) first, then this half's (kept)
//   dP^T = V dO_j^T   -> TMEM [128,256)   this half's dO sub-tiles first, then the other half's
//   elementwise: P^T = exp2(S^T * scale_log2 - LSE2[q]) (masked on PARTIAL tiles),
//                dS^T = P^T * (dP^T - Dsum[q]); both written over their own columns as bf16 pairs
//   dV_h += P^T dO_j[:, h]  -> TMEM [256,384)   A = P^T (TMEM), B = dO half (MN-major)
//   dK_h += dS^T Q_j[:, h]  -> TMEM [384,512)   A = dS^T (TMEM), B = Q half (MN-major)
// At the end dK_h (x scale) and dV_h are added by TMA tensor reductions into fp32 per-KV-head
// accumulators (the GQA group's query heads are separate CTAs).
// =================================================================================================
struct KvParams {
  float *dk_acc, *dv_acc;   // [B, T, Hkv, D] fp32, pre-zeroed
  const float *lse, *dsum;  // [B, Hq, T]
  const int16_t* list;      // [B, nk, nq] entries qt | cls << 14
  const int* cnt;           // [B, nk]
  const uint4* tmask_t;     // [B, nk, nq, 128] column masks of PARTIAL tiles (bit q = query q allowed)
  int* err;
  int T, Hq, group, nq, B;
  float scale, scale_log2;
};

struct KvSmem {
  static constexpr int K = 0;                 // 4 sub-tiles
  static constexpr int V = K + 4 * SUB;       // 4 sub-tiles
  static constexpr int OWN = V + 4 * SUB;     // Q_j[:, h] (2 sub-tiles) then dO_j[:, h] (2 sub-tiles)
  static constexpr int TR = OWN + 4 * SUB;    // 2 transient sub-tile slots (the other half of Q_j, dO_j)
  static constexpr int LSE = TR + 2 * SUB;    // float[128]
  static constexpr int DS = LSE + 512;        // float[128]
  static constexpr int BAR = DS + 512;
  static constexpr int TOTAL = BAR + 256;
};
static_assert(KvSmem::TOTAL + 1024 <= 232448, "dK / dV shared memory");

__global__ void __launch_bounds__(NTH, 1)
    bwd_kv_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                  const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                  const __grid_constant__ CUtensorMap tmDK, const __grid_constant__ CUtensorMap tmDV,
                  const KvParams p) {
  using S = KvSmem;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::BAR);
  uint64_t* kv_full = bars + 0;
  uint64_t* own_full = bars + 1;
  uint64_t* own_empty = bars + 2;
  uint64_t* tr_full = bars + 3;     // [2]
  uint64_t* tr_empty = bars + 5;    // [2]
  uint64_t* sp_full = bars + 7;
  uint64_t* p_full = bars + 8;
  uint64_t* mma_done = bars + 9;    // every MMA of the pair has completed
  uint64_t* drain = bars + 10;
  uint64_t* fin = bars + 11;        // every MMA of the CTA has completed (the epilogue's single phase)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);
  float* sLSE = reinterpret_cast<float*>(smem + S::LSE);
  float* sDs = reinterpret_cast<float*>(smem + S::DS);

  const int kt = blockIdx.x, h = blockIdx.y, b = blockIdx.z >> 1, hf = blockIdx.z & 1, oh = hf ^ 1;
  const int hk = h / p.group;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = gridDim.x;
  const int lidx = b * nk + kt;
  const int total = p.cnt[lidx];
  const int16_t* list = p.list + (int64_t)lidx * p.nq;
  // neighbouring key tiles start their walk at different query tiles
  const int rot = total > 0 ? (kt * 7 + h * 3) % total : 0;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    mbar_init(own_full, 1);
    mbar_init(own_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tr_full[i], 1);
      mbar_init(&tr_empty[i], 1);
    }
    mbar_init(sp_full, 1);
    mbar_init(p_full, 256);
    mbar_init(mma_done, 1);
    mbar_init(drain, 1);
    mbar_init(fin, 1);
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tDP = tmem + 128, tDV = tmem + 256, tDK = tmem + 384;

  if (warp == 9) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      prefetch_tmap(&tmDO);
      mbar_expect_tx(kv_full, 8 * SUB);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        tma_load_4d(smem + S::K + c * SUB, &tmK, kv_full, c * 64, hk, kt * BM, b);
        tma_load_4d(smem + S::V + c * SUB, &tmV, kv_full, c * 64, hk, kt * BM, b);
      }
      int u = 0;
      // one transient sub-tile: column block c of `map` for query tile qt
      auto transient = [&](const CUtensorMap* map, int c, int qt) {
        const int slot = u & 1;
        if (u >= 2 && !mbar_wait(&tr_empty[slot], ((u >> 1) - 1) & 1, p.err, 41)) return false;
        mbar_expect_tx(&tr_full[slot], SUB);
        tma_load_4d(smem + S::TR + slot * SUB, map, &tr_full[slot], c * 64, h, qt * BM, b);
        ++u;
        return true;
      };
      bool ok = true;
      for (int j = 0; ok && j < total; ++j) {
        const int qt = list[(j + rot) % total] & 0x3fff;
        ok = transient(&tmQ, 2 * oh, qt) && transient(&tmQ, 2 * oh + 1, qt);
        if (!ok) break;
        // this half's Q / dO sub-tiles: the slot held pair j-1's, read by its dV / dK MMAs
        if (j >= 1 && !(ok = mbar_wait(own_empty, (j - 1) & 1, p.err, 42))) break;
        mbar_expect_tx(own_full, 4 * SUB);
        for (int c = 0; c < 2; ++c) {
          tma_load_4d(smem + S::OWN + c * SUB, &tmQ, own_full, (2 * hf + c) * 64, h, qt * BM, b);
          tma_load_4d(smem + S::OWN + (2 + c) * SUB, &tmDO, own_full, (2 * hf + c) * 64, h, qt * BM, b);
        }
        ok = transient(&tmDO, 2 * oh, qt) && transient(&tmDO, 2 * oh + 1, qt);
      }
      // the last loads must have landed before the CTA can retire
      if (ok && total > 0) {
        mbar_wait(own_full, (total - 1) & 1, p.err, 43);
        for (int v = u - 2; v < u; ++v) mbar_wait(&tr_full[v & 1], (v >> 1) & 1, p.err, 43);
      }
    }
  } else if (warp == 8) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idKK = idesc_bf16_f32(128, 128, 0, 0);   // S^T, dP^T
      constexpr uint32_t idKM = idesc_bf16_f32(128, 128, 0, 1);   // dV_h, dK_h (B MN-major)
      const uint32_t sK = smem_addr(smem + S::K), sV = smem_addr(smem + S::V), sOwn = smem_addr(smem + S::OWN),
                     sTR = smem_addr(smem + S::TR);
      bool ok = mbar_wait(kv_full, 0, p.err, 44);
      int u = 0;
      // 4 K-steps of 16 over one 64-column block: A = sub-tile `a` of K or V, B = `bsub`
      auto steps = [&](uint32_t acc_tmem, uint32_t a, uint32_t bsub, bool first) {
#pragma unroll
        for (int k = 0; k < 4; ++k)
          umma_f16(acc_tmem, desc_sw128(a + k * 32, 16, 1024), desc_sw128(bsub + k * 32, 16, 1024), idKK,
                   (first && k == 0) ? 0u : 1u);
      };
      auto take_transient = [&](uint32_t acc_tmem, uint32_t a, bool first) {
        const int slot = u & 1;
        if (!mbar_wait(&tr_full[slot], (u >> 1) & 1, p.err, 45)) return false;
        tc_fence_after();
        steps(acc_tmem, a, sTR + slot * SUB, first);
        umma_commit(&tr_empty[slot]);
        ++u;
        return true;
      };
      for (int j = 0; ok && j < total; ++j) {
        // S^T_j goes over P^T_{j-1}, dP^T_j over dS^T_{j-1}: pair j-1's dV / dK MMAs must have run
        if (j > 0 && !(ok = mbar_wait(mma_done, (j - 1) & 1, p.err, 46))) break;
        tc_fence_after();
        if (!(ok = take_transient(tS, sK + (2 * oh) * SUB, true))) break;
        if (!(ok = take_transient(tS, sK + (2 * oh + 1) * SUB, false))) break;
        if (!(ok = mbar_wait(own_full, j & 1, p.err, 47))) break;
        tc_fence_after();
        steps(tS, sK + (2 * hf) * SUB, sOwn, false);
        steps(tS, sK + (2 * hf + 1) * SUB, sOwn + SUB, false);
        steps(tDP, sV + (2 * hf) * SUB, sOwn + 2 * SUB, true);
        steps(tDP, sV + (2 * hf + 1) * SUB, sOwn + 3 * SUB, false);
        if (!(ok = take_transient(tDP, sV + (2 * oh) * SUB, false))) break;
        if (!(ok = take_transient(tDP, sV + (2 * oh + 1) * SUB, false))) break;
        umma_commit(sp_full);
        if (!(ok = mbar_wait(p_full, j & 1, p.err, 48))) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          // queries [16 kk, 16 kk + 16): written by group kk / 4 at column 64 (kk / 4) + 8 (kk % 4)
          const uint32_t acol = (kk >> 2) * 64 + (kk & 3) * 8;
          const uint32_t acc = (j > 0 || kk > 0) ? 1u : 0u;
          umma_f16_ts(tDV, tS + acol, desc_sw128(sOwn + 2 * SUB + kk * 2048, SUB, 1024), idKM, acc);
          umma_f16_ts(tDK, tDP + acol, desc_sw128(sOwn + kk * 2048, SUB, 1024), idKM, acc);
        }
        umma_commit(own_empty);
        umma_commit(mma_done);
      }
      if (ok) umma_commit(fin);
      umma_commit(drain);
      mbar_wait(drain, 0, p.err, 49);
    }
  } else {
    // ---------------- warps 0-7: P^T and dS^T ----------------
    const int r = threadIdx.x & 127, g = threadIdx.x >> 7;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    bool ok = true;
    // the next pair's list entry, -LSE2 / -Dsum of its query row r and PARTIAL-tile mask are
    // loaded one pair ahead
    int e_next = total > 0 ? list[rot % total] : 0;
    float lse_next = -INFINITY, ds_next = 0.f;
    uint2 cm_next = make_uint2(0xffffffffu, 0xffffffffu);
    auto fetch = [&](int e) {
      const int qn = (e & 0x3fff) * 128 + r;
      if (g == 0) {
        const int64_t li = ((int64_t)b * p.Hq + h) * p.T + qn;
        lse_next = qn < p.T ? -p.lse[li] * 1.44269504088896340736f : -INFINITY;
        ds_next = qn < p.T ? -p.dsum[li] : 0.f;
      }
      cm_next = make_uint2(0xffffffffu, 0xffffffffu);
      if ((e >> 14) != CLS_FULL) {
        const uint4 m4 = p.tmask_t[(((int64_t)b * nk + kt) * p.nq + (e & 0x3fff)) * 128 + r];
        cm_next = g == 0 ? make_uint2(m4.x, m4.y) : make_uint2(m4.z, m4.w);
      }
    };
    if (total > 0) fetch(e_next);
    for (int j = 0; j < total; ++j) {
      const uint2 cm = cm_next;
      if (g == 0) {
        sLSE[r] = lse_next;
        sDs[r] = ds_next;
      }
      if (j + 1 < total) e_next = list[(j + 1 + rot) % total];
      named_bar_sync_256();
      if (ok) ok = mbar_wait(sp_full, j & 1, p.err, 50);
      tc_fence_after();
      if (j + 1 < total) fetch(e_next);
      if (ok) {
        uint32_t sv[2][16], dv[2][16];
        tmem_ld16(tS + lane_off + g * 64, sv[0]);
        tmem_ld16(tDP + lane_off + g * 64, dv[0]);
        const uint64_t scale2 = f2pack(p.scale_log2, p.scale_log2);
#pragma unroll
        for (int sc = 0; sc < 4; ++sc) {
          const int cur = sc & 1;
          const int q0 = g * 64 + sc * 16;
          tmem_wait_ld();
          if (sc < 3) {
            tmem_ld16(tS + lane_off + q0 + 16, sv[cur ^ 1]);
            tmem_ld16(tDP + lane_off + q0 + 16, dv[cur ^ 1]);
          }
          const uint32_t amask = ((sc < 2 ? cm.x : cm.y) >> ((sc & 1) * 16)) & 0xffffu;
          uint32_t pw[8], dw[8];
#pragma unroll
          for (int t4 = 0; t4 < 4; ++t4) {
            const float4 l4 = reinterpret_cast<const float4*>(sLSE + q0)[t4];
            const float4 d4 = reinterpret_cast<const float4*>(sDs + q0)[t4];
#pragma unroll
            for (int u2 = 0; u2 < 2; ++u2) {
              const int t = t4 * 4 + u2 * 2;
              const uint64_t x = f2fma(f2pack(__uint_as_float(sv[cur][t]), __uint_as_float(sv[cur][t + 1])), scale2,
                                       u2 == 0 ? f2pack(l4.x, l4.y) : f2pack(l4.z, l4.w));
              const float2 xf = f2unpack(x);
              float e0 = fast_exp2(xf.x), e1 = fast_exp2(xf.y);
              if (amask != 0xffffu) {
                e0 = ((amask >> t) & 1u) ? e0 : 0.f;
                e1 = ((amask >> (t + 1)) & 1u) ? e1 : 0.f;
              }
              const uint64_t dd = f2mul(f2pack(e0, e1),
                                        f2add(f2pack(__uint_as_float(dv[cur][t]), __uint_as_float(dv[cur][t + 1])),
                                              u2 == 0 ? f2pack(d4.x, d4.y) : f2pack(d4.z, d4.w)));
              const float2 df = f2unpack(dd);
              const __nv_bfloat162 pb = __floats2bfloat162_rn(e0, e1);
              const __nv_bfloat162 db = __floats2bfloat162_rn(df.x, df.y);
              pw[t >> 1] = *reinterpret_cast<const uint32_t*>(&pb);
              dw[t >> 1] = *reinterpret_cast<const uint32_t*>(&db);
            }
          }
          // P^T / dS^T (bf16 pairs) over columns [64 g + 8 sc, 64 g + 8 sc + 8) of S^T / dP^T,
          // whose values were loaded with sub-chunk sc / 2
          tmem_st8(tS + lane_off + g * 64 + sc * 8, pw);
          tmem_st8(tDP + lane_off + g * 64 + sc * 8, dw);
        }
        tmem_wait_st();
      }
      tc_fence_before();
      named_bar_sync_256();        // every thread has read this pair's LSE / Dsum
      mbar_arrive(p_full);
    }
    if (ok && total > 0) ok = mbar_wait(fin, 0, p.err, 51);
    named_bar_sync_256();
    // dK_h (x scale) and dV_h staged as fp32 [128 rows][32] 128B-swizzled chunks in the idle Q / dO
    // slots, then added by TMA into the fp32 accumulators at columns [128 hf, 128 hf + 128) (rows
    // past T are clipped).  The barrier sequence depends only on `total` (uniform); a thread whose
    // wait timed out skips the data movement.
    if (total > 0) {
      tc_fence_after();
      unsigned char* stage = smem + S::OWN;
#pragma unroll 1
      for (int which = 0; which < 2; ++which) {
        const uint32_t src = which == 0 ? tDK : tDV;
        const float mul = which == 0 ? p.scale : 1.f;
        if (ok) {
#pragma unroll 1
          for (int cc = 0; cc < 2; ++cc) {
            const int c = g * 2 + cc;
            uint32_t t[32];
            tmem_ld32(src + lane_off + c * 32, t);
            tmem_wait_ld();
            unsigned char* sc = stage + c * SUB;
#pragma unroll
            for (int u = 0; u < 8; ++u)
              *reinterpret_cast<float4*>(sc + r * 128 + ((u ^ (r & 7)) << 4)) =
                  make_float4(__uint_as_float(t[u * 4]) * mul, __uint_as_float(t[u * 4 + 1]) * mul,
                              __uint_as_float(t[u * 4 + 2]) * mul, __uint_as_float(t[u * 4 + 3]) * mul);
          }
        }
        fence_async_smem();
        named_bar_sync_256();
        if (threadIdx.x == 0 && ok) {
#pragma unroll 1
          for (int c = 0; c < 4; ++c)
            attn100::tma_reduce_add_4d(which == 0 ? &tmDK : &tmDV, stage + c * SUB, hf * 128 + c * 32, hk, kt * BM, b);
          attn100::bulk_commit();
          attn100::bulk_wait_read();
        }
        named_bar_sync_256();
      }
    }
    if (threadIdx.x == 0) attn100::bulk_wait_all();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

// =================================================================================================
// Backward, dQ.  CTA = (128-query tile qt, query head h); it walks the forward list of the query
// tile (thread (g, r) owns query row r == TMEM lane r and key columns [64 g, 64 g + 64)):
//   S_i  = Q K_i^T    -> TMEM [0,128)     A = Q (resident), B = K_i (kept until dQ_i has run)
//   dP_i = dO V_i^T   -> TMEM [128,256)   A = dO (resident), B = V_i through two transient slots
//   elementwise: dS = exp2(S * scale_log2 - LSE2) * (dP - Dsum), masked, written over S as bf16
//   dQ  += dS K_i     -> TMEM [256,512)   A = dS (TMEM), B = K_i (MN-major), two N = 128 halves
// dQ (x scale) is complete after the last key tile: it leaves as bf16 through the Q tile by TMA.
// =================================================================================================
struct QParams {
  const float *lse, *dsum;  // [B, Hq, T]
  const int16_t* list;      // [B, nq, nk] entries kt | cls << 14
  const int* cnt;           // [B, nq]
  const uint4* tmask;       // [B, nq, nk, 128] row masks of PARTIAL tiles
  int* err;
  int T, Hq, group, nk;
  float scale, scale_log2;
};

struct QSmem {
  static constexpr int Q = 0;                 // 4 sub-tiles (the dQ staging tile at the end)
  static constexpr int DO = Q + 4 * SUB;      // 4 sub-tiles
  static constexpr int KB = DO + 4 * SUB;     // K_i, 4 sub-tiles
  static constexpr int TR = KB + 4 * SUB;     // 2 transient slots (V_i)
  static constexpr int BAR = TR + 2 * SUB;
  static constexpr int TOTAL = BAR + 256;
};
static_assert(QSmem::TOTAL + 1024 <= 232448, "dQ shared memory");

__global__ void __launch_bounds__(NTH, 1)
    bwd_q_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                 const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                 const __grid_constant__ CUtensorMap tmDQ, const QParams p) {
  using S = QSmem;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::BAR);
  uint64_t* qd_full = bars + 0;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = bars + 2;
  uint64_t* tr_full = bars + 3;     // [2]
  uint64_t* tr_empty = bars + 5;    // [2]
  uint64_t* sp_full = bars + 7;
  uint64_t* p_full = bars + 8;
  uint64_t* fin = bars + 9;         // every MMA of the CTA has completed
  uint64_t* drain = bars + 10;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 11);

  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int hk = h / p.group;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nq = gridDim.x;
  const int lidx = b * nq + qt;
  const int n = p.cnt[lidx];
  const int16_t* list = p.list + (int64_t)lidx * p.nk;

  if (threadIdx.x == 0) {
    mbar_init(qd_full, 1);
    mbar_init(k_full, 1);
    mbar_init(k_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tr_full[i], 1);
      mbar_init(&tr_empty[i], 1);
    }
    mbar_init(sp_full, 1);
    mbar_init(p_full, 256);
    mbar_init(fin, 1);
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tDP = tmem + 128, tDQ = tmem + 256;

  if (warp == 9) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      prefetch_tmap(&tmDO);
      mbar_expect_tx(qd_full, 8 * SUB);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        tma_load_4d(smem + S::Q + c * SUB, &tmQ, qd_full, c * 64, h, qt * BM, b);
        tma_load_4d(smem + S::DO + c * SUB, &tmDO, qd_full, c * 64, h, qt * BM, b);
      }
      int u = 0;
      auto transient = [&](int c, int kt) {
        const int slot = u & 1;
        if (u >= 2 && !mbar_wait(&tr_empty[slot], ((u >> 1) - 1) & 1, p.err, 61)) return false;
        mbar_expect_tx(&tr_full[slot], SUB);
        tma_load_4d(smem + S::TR + slot * SUB, &tmV, &tr_full[slot], c * 64, hk, kt * BM, b);
        ++u;
        return true;
      };
      bool ok = true;
      for (int i = 0; ok && i < n; ++i) {
        const int kt = list[i] & 0x3fff;
        // V_i's first two sub-tiles need only transient slots; K_i waits for dQ_{i-1}
        if (!(ok = transient(0, kt) && transient(1, kt))) break;
        if (i >= 1 && !(ok = mbar_wait(k_empty, (i - 1) & 1, p.err, 62))) break;
        mbar_expect_tx(k_full, 4 * SUB);
#pragma unroll
        for (int c = 0; c < 4; ++c) tma_load_4d(smem + S::KB + c * SUB, &tmK, k_full, c * 64, hk, kt * BM, b);
        ok = transient(2, kt) && transient(3, kt);
      }
      if (ok && n > 0) {
        mbar_wait(k_full, (n - 1) & 1, p.err, 63);
        for (int v = u - 2; v < u; ++v) mbar_wait(&tr_full[v & 1], (v >> 1) & 1, p.err, 63);
      }
    }
  } else if (warp == 8) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idKK = idesc_bf16_f32(128, 128, 0, 0);   // S, dP
      constexpr uint32_t idKM = idesc_bf16_f32(128, 128, 0, 1);   // dQ halves (B MN-major)
      const uint32_t sQ = smem_addr(smem + S::Q), sDO = smem_addr(smem + S::DO), sKB = smem_addr(smem + S::KB),
                     sTR = smem_addr(smem + S::TR);
      bool ok = mbar_wait(qd_full, 0, p.err, 64);
      int u = 0;
      for (int i = 0; ok && i < n; ++i) {
        // K_i has landed, so dQ_{i-1} (which read dS_{i-1} from TMEM [0,128)) has completed
        if (!(ok = mbar_wait(k_full, i & 1, p.err, 65))) break;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          const uint32_t off = (k >> 2) * SUB + (k & 3) * 32;
          umma_f16(tS, desc_sw128(sQ + off, 16, 1024), desc_sw128(sKB + off, 16, 1024), idKK, k > 0 ? 1u : 0u);
        }
        for (int c = 0; c < 4; ++c, ++u) {
          const int slot = u & 1;
          if (!(ok = mbar_wait(&tr_full[slot], (u >> 1) & 1, p.err, 66))) break;
          tc_fence_after();
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_f16(tDP, desc_sw128(sDO + c * SUB + k * 32, 16, 1024), desc_sw128(sTR + slot * SUB + k * 32, 16, 1024),
                     idKK, (c > 0 || k > 0) ? 1u : 0u);
          umma_commit(&tr_empty[slot]);
        }
        if (!ok) break;
        umma_commit(sp_full);
        if (!(ok = mbar_wait(p_full, i & 1, p.err, 67))) break;
        tc_fence_after();
#pragma unroll
        for (int hh = 0; hh < 2; ++hh)
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            // keys [16 kk, 16 kk + 16): dS written by group kk / 4 at column 64 (kk / 4) + 8 (kk % 4)
            umma_f16_ts(tDQ + hh * 128, tS + (kk >> 2) * 64 + (kk & 3) * 8,
                        desc_sw128(sKB + hh * 2 * SUB + kk * 2048, SUB, 1024), idKM, (i > 0 || kk > 0) ? 1u : 0u);
        umma_commit(k_empty);
      }
      if (ok) umma_commit(fin);
      umma_commit(drain);
      mbar_wait(drain, 0, p.err, 68);
    }
  } else {
    // ---------------- warps 0-7: dS ----------------
    const int r = threadIdx.x & 127, g = threadIdx.x >> 7;
    const int row = qt * BM + r;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const int64_t li = ((int64_t)b * p.Hq + h) * p.T + row;
    const float nlse2 = row < p.T ? -p.lse[li] * 1.44269504088896340736f : -INFINITY;
    const float ndsum = row < p.T ? -p.dsum[li] : 0.f;
    const uint64_t l2 = f2pack(nlse2, nlse2), d2 = f2pack(ndsum, ndsum), scale2 = f2pack(p.scale_log2, p.scale_log2);
    bool ok = true;
    for (int i = 0; i < n; ++i) {
      const int entry = list[i];
      const int kt = entry & 0x3fff;
      uint2 cm = make_uint2(0xffffffffu, 0xffffffffu);
      if ((entry >> 14) != CLS_FULL) {
        const uint4 w = p.tmask[(((int64_t)b * nq + qt) * p.nk + kt) * BM + r];
        cm = g == 0 ? make_uint2(w.x, w.y) : make_uint2(w.z, w.w);
      }
      if (ok) ok = mbar_wait(sp_full, i & 1, p.err, 69);
      tc_fence_after();
      if (ok) {
        uint32_t sv[2][16], dv[2][16];
        tmem_ld16(tS + lane_off + g * 64, sv[0]);
        tmem_ld16(tDP + lane_off + g * 64, dv[0]);
#pragma unroll
        for (int sc = 0; sc < 4; ++sc) {
          const int cur = sc & 1;
          const int k0 = g * 64 + sc * 16;
          tmem_wait_ld();
          if (sc < 3) {
            tmem_ld16(tS + lane_off + k0 + 16, sv[cur ^ 1]);
            tmem_ld16(tDP + lane_off + k0 + 16, dv[cur ^ 1]);
          }
          const uint32_t amask = ((sc < 2 ? cm.x : cm.y) >> ((sc & 1) * 16)) & 0xffffu;
          uint32_t dw[8];
#pragma unroll
          for (int t = 0; t < 16; t += 2) {
            const float2 xf =
                f2unpack(f2fma(f2pack(__uint_as_float(sv[cur][t]), __uint_as_float(sv[cur][t + 1])), scale2, l2));
            float e0 = fast_exp2(xf.x), e1 = fast_exp2(xf.y);
            if (amask != 0xffffu) {
              e0 = ((amask >> t) & 1u) ? e0 : 0.f;
              e1 = ((amask >> (t + 1)) & 1u) ? e1 : 0.f;
            }
            const float2 df = f2unpack(
                f2mul(f2pack(e0, e1), f2add(f2pack(__uint_as_float(dv[cur][t]), __uint_as_float(dv[cur][t + 1])), d2)));
            const __nv_bfloat162 db = __floats2bfloat162_rn(df.x, df.y);
            dw[t >> 1] = *reinterpret_cast<const uint32_t*>(&db);
          }
          tmem_st8(tS + lane_off + g * 64 + sc * 8, dw);
        }
        tmem_wait_st();
      }
      tc_fence_before();
      mbar_arrive(p_full);
    }
    if (ok && n > 0) ok = mbar_wait(fin, 0, p.err, 70);
    // dQ (x scale) as bf16 in the idle Q tile (every S MMA has completed), stored by TMA; a query
    // tile without key tiles stores zeros
    unsigned char* sO = smem + S::Q;
    if (ok) {
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t t[32];
        if (n > 0) {
          tmem_ld32(tDQ + lane_off + g * 128 + c * 32, t);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) t[j] = 0u;
        }
#pragma unroll
        for (int j8 = 0; j8 < 4; ++j8) {
          float f[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) f[j] = __uint_as_float(t[j8 * 8 + j]) * p.scale;
          const int col = g * 128 + c * 32 + j8 * 8;
          store8(reinterpret_cast<bf16*>(sO + (col >> 6) * SUB + sw128_offset(r, col & 63)), f);
        }
      }
      fence_async_smem();
    }
    named_bar_sync_256();
    if (threadIdx.x == 0 && ok) {
#pragma unroll
      for (int c = 0; c < 4; ++c) attn100::tma_store_4d(&tmDQ, sO + c * SUB, c * 64, h, qt * BM, b);
      attn100::bulk_commit();
      attn100::bulk_wait_all();
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

template <typename Kern>
static void allow_smem(Kern kern, int bytes) {
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

}  // namespace attn256

using attn100::make_map;
using attn100::make_map_f32;

int bd_attn_fwd_d256(const AttnTensors& t, const int16_t* list128, const int* cnt128, const uint4* rowmask,
                     const int4* meta, int flags, float scale, int* err, cudaStream_t s) {
  if (t.D != 256) return -1;
  attn256::FwdParams p;
  p.lse = t.lse; p.meta = meta; p.list = list128; p.cnt = cnt128; p.tmask = rowmask; p.err = err;
  p.T = t.T; p.Hq = t.Hq; p.group = t.Hq / t.Hkv; p.nk = (t.T + 127) / 128; p.flags = flags;
  p.scale_log2 = scale * 1.44269504088896340736f;
  CUtensorMap mq, mk, mv, mo;
  if (!make_map(&mq, t.q, t.B, t.T, t.Hq, 256, t.q_tok, t.q_b)) return -2;
  if (!make_map(&mk, t.k, t.B, t.T, t.Hkv, 256, t.k_tok, t.k_b)) return -3;
  if (!make_map(&mv, t.v, t.B, t.T, t.Hkv, 256, t.v_tok, t.v_b)) return -4;
  if (!make_map(&mo, t.o, t.B, t.T, t.Hq, 256, t.o_tok, t.o_b)) return -5;
  const int smem = attn256::FwdSmem::TOTAL + 1024;
  static bool init = false;
  if (!init) {
    attn256::allow_smem(attn256::fwd_kernel, smem);
    init = true;
  }
  const int nq = (t.T + 127) / 128;
  attn256::fwd_kernel<<<dim3(nq, t.Hq, t.B), attn256::NTH, smem, s>>>(mq, mk, mv, mo, p);
  return 0;
}

int bd_attn_bwd_d256(const AttnTensors& t, const bf16* dout, int64_t do_tok, int64_t do_b, const float* dsum,
                     float* dk_acc, float* dv_acc, bf16* dq, int64_t dq_tok, int64_t dq_b, const int16_t* list128t,
                     const int* cnt128t, const uint4* colmask, const int16_t* list128, const int* cnt128,
                     const uint4* rowmask, float scale, int* err, cudaStream_t s) {
  if (t.D != 256) return -1;
  const int nq = (t.T + 127) / 128, nk = nq;
  CUtensorMap mq, mk, mv, mdo, mdk, mdv, mdq;
  if (!make_map(&mq, t.q, t.B, t.T, t.Hq, 256, t.q_tok, t.q_b)) return -2;
  if (!make_map(&mk, t.k, t.B, t.T, t.Hkv, 256, t.k_tok, t.k_b)) return -3;
  if (!make_map(&mv, t.v, t.B, t.T, t.Hkv, 256, t.v_tok, t.v_b)) return -4;
  if (!make_map(&mdo, dout, t.B, t.T, t.Hq, 256, do_tok, do_b)) return -5;
  if (!make_map(&mdq, dq, t.B, t.T, t.Hq, 256, dq_tok, dq_b)) return -6;
  if (!make_map_f32(&mdk, dk_acc, t.B, t.T, t.Hkv, 256)) return -7;
  if (!make_map_f32(&mdv, dv_acc, t.B, t.T, t.Hkv, 256)) return -8;

  attn256::KvParams kp;
  kp.dk_acc = dk_acc; kp.dv_acc = dv_acc; kp.lse = t.lse; kp.dsum = dsum; kp.list = list128t; kp.cnt = cnt128t;
  kp.tmask_t = colmask; kp.err = err; kp.T = t.T; kp.Hq = t.Hq; kp.group = t.Hq / t.Hkv; kp.nq = nq; kp.B = t.B;
  kp.scale = scale; kp.scale_log2 = scale * 1.44269504088896340736f;
  attn256::QParams qp;
  qp.lse = t.lse; qp.dsum = dsum; qp.list = list128; qp.cnt = cnt128; qp.tmask = rowmask; qp.err = err;
  qp.T = t.T; qp.Hq = t.Hq; qp.group = t.Hq / t.Hkv; qp.nk = nk;
  qp.scale = scale; qp.scale_log2 = kp.scale_log2;

  const int smem_kv = attn256::KvSmem::TOTAL + 1024, smem_q = attn256::QSmem::TOTAL + 1024;
  static bool init = false;
  if (!init) {
    attn256::allow_smem(attn256::bwd_kv_kernel, smem_kv);
    attn256::allow_smem(attn256::bwd_q_kernel, smem_q);
    init = true;
  }
  attn256::bwd_kv_kernel<<<dim3(nk, t.Hq, 2 * t.B), attn256::NTH, smem_kv, s>>>(mq, mk, mv, mdo, mdk, mdv, kp);
  attn256::bwd_q_kernel<<<dim3(nq, t.Hq, t.B), attn256::NTH, smem_q, s>>>(mq, mk, mv, mdo, mdq, qp);
  return 0;
}

}  // namespace trida
