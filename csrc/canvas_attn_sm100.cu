// Serving canvas attention on the 5th-generation tensor cores (head_dim 128 / 256).
//
// A self-speculative decode step attends every canvas row of a request to that request's cached
// prefix and to the canvas itself: the first n_clean canvas rows are token-causal, the remaining
// (MASK) rows see the whole canvas, and every row sees the whole prefix.  The canvas K / V rows are
// appended to the cache first (kv_append), so all keys come from the cache: positions [0, pos + blk).
// Behaviour follows the reference's canvas rule (inference/zoro-1/mlx/trida_mlx/model.py:461-470 and
// the vLLM self-spec backend's draft/verify attention, vllm_native_diffusion/qwen3_5_diffusion.py).
//
// Tiling.  CTA = (128 query rows, one KV head, one request, one key split).  The 128 rows are the GQA
// group's G query heads x 128/G canvas rows, ordered (canvas row, head): q is [rows, Hq, D], so one
// 4-D TMA box {64 columns, G heads, 128/G rows} per 64-column sub-tile gathers the whole query tile
// (rows past the request's canvas belong to the next request or lie past the tensor; they are
// computed and never stored).  Keys move in tiles of 128 positions = two 64-position cache pages, one
// TMA box per page, so a paged cache needs no gather kernel: the page table is read by the producer
// thread and only changes the box coordinates.  Pages past the table are loaded from a row past the
// tensor (TMA fills zeros), so every V row an MMA reads is finite.
//
//   TMEM = S0 | S1 | O (128 + 128 + D columns of 512): S = Q K^T contracts over D in 16-column steps
//   (A = Q in shared memory, K-major), P is written over S as bf16 pairs and is the TMEM A operand of
//   O += P V (V MN-major in shared memory).  Softmax of tile i overlaps S_{i+1}; O is rescaled in TMEM
//   only when a row's max grows by more than 2^16 (lazy rescaling).
//   Warps 0-7: softmax (thread (half, r) owns TMEM lane r and 64 of the tile's 128 key columns),
//   warp 8: MMA issue (one thread), warp 9: TMA loads (one thread).  Every wait is bounded and records
//   an error code in the device error word instead of hanging.
//
// Output.  One key split: O / l is written as bf16 rows of out [rows, Hq, D] straight from TMEM.
// Several splits (few requests): unnormalised fp32 partial rows plus (max, sum) per row, merged by
// the combine kernel in serve.cu.
#include <cudaTypedefs.h>

#include <algorithm>
#include <climits>

#include "common.cuh"
#include "ops.h"
#include "sm100_common.cuh"
#include "bd_attention_sm100.cuh"

namespace trida {
namespace canvas100 {

using namespace sm100;
using attn100::fast_exp2;
using attn100::named_sync;
using attn100::RESCALE_THRESHOLD;

constexpr int BM = 128;          // query rows per CTA (TMEM lanes)
constexpr int BN = 128;          // keys per tile
constexpr int PAGE = 64;         // positions per cache page (one TMA box of keys)
constexpr int SUB = 128 * 128;   // bytes of a [128 rows][64 bf16] swizzled sub-tile
constexpr int NTH = 320;         // 8 softmax warps + MMA warp + TMA warp
constexpr int RING = 5;          // K / V ring of units (a unit = two sub-tiles = 128 d-columns x 128 keys)

struct Params {
  const int* slot;   // [B] cache slot of each request
  const int* pos;    // [B] cached prefix length (the canvas keys start there)
  const int* ptab;   // paged cache: [slots, maxpages] page of every 64 positions; null: dense cache
  bf16* out;         // [B * blk, Hq, D] (one split)
  float* po;         // [B, nsplit, Hq, blk, D] unnormalised partial outputs (several splits)
  float* pm;         // [B, nsplit, Hq, blk] running max (scaled, log2 domain; -inf: no visible key)
  float* pl;         // [B, nsplit, Hq, blk] running sum
  int* err;
  int maxpages, maxlen, cache_rows;   // cache_rows: rows of the cache's 2-D view (a row past it reads zeros)
  int n_slots;                        // rows of the page table (paged) or slots of the dense cache
  int blk, n_clean, Hq, G, rpt, nqt, nsplit, tps;   // rpt = canvas rows per tile, tps = key tiles per split
  float scale_log2;
};

template <int D>
struct Smem {
  static constexpr int Q = 0;                          // D / 64 sub-tiles
  static constexpr int R0 = Q + (D / 64) * SUB;        // K / V unit ring
  static constexpr int XCH = R0 + RING * 2 * SUB;      // half-row max / sum exchange
  static constexpr int BAR = XCH + 2 * BM * 4;
  static constexpr int TOTAL = BAR + 256;
};
static_assert(Smem<256>::TOTAL + 1024 <= 232448, "canvas attention shared memory");

template <int D>
__global__ void __launch_bounds__(NTH, 1)
    canvas_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                  const __grid_constant__ CUtensorMap tmV, const Params p) {
  constexpr int NU = D / 128;    // K / V units per key tile
  constexpr int NQS = D / 64;    // Q sub-tiles
  using S = Smem<D>;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::BAR);
  uint64_t* q_full = bars + 0;
  uint64_t* u_full = bars + 1;               // [RING]
  uint64_t* u_empty = bars + 1 + RING;       // [RING]
  uint64_t* s_full = bars + 1 + 2 * RING;    // [2]
  // [2]: P_i written completes p_full[i & 1].  One barrier per tile parity: S_{i+1} is issued before
  // PV_i, so a softmax warp can finish tile i+1 while another is still on tile i, and with a single
  // 256-arrival barrier its early arrival would complete tile i's phase before every P_i is written.
  // It cannot get two tiles ahead (S_{i+2} waits for PV_i, which waits for all of tile i).
  uint64_t* p_full = s_full + 2;
  uint64_t* pv_done = p_full + 2;            // [2]
  uint64_t* drain = pv_done + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int split = blockIdx.x, b = blockIdx.z;
  const int qt = blockIdx.y % p.nqt, hk = blockIdx.y / p.nqt;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int slot = p.slot[b], pos = p.pos[b];
  // a slot or position outside the cache is recorded (code 220) and the request is skipped: no
  // page-table read, no load and no store with a bad index
  const bool valid = slot >= 0 && slot < p.n_slots && pos >= 0 && pos <= p.maxlen - p.blk;
  if (!valid && threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0) atomicCAS(p.err, 0, 220);
  const int kend = pos + p.blk;                        // keys [0, kend)
  const int ntile = (kend + BN - 1) / BN;
  const int t0 = split * p.tps;
  const int n = valid ? max(0, min(ntile, t0 + p.tps) - t0) : 0;   // key tiles of this split

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
    if (lane == 0 && n > 0) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      mbar_expect_tx(q_full, NQS * SUB);
#pragma unroll
      for (int c = 0; c < NQS; ++c)
        tma_load_4d(smem + S::Q + c * SUB, &tmQ, q_full, c * 64, hk * p.G, b * p.blk + qt * p.rpt, 0);
      // cache row of the first position of page `pg` of this request (a row past the view: zeros)
      auto page_row = [&](int pg) -> int {
        if (p.ptab != nullptr) return pg < p.maxpages ? p.ptab[(int64_t)slot * p.maxpages + pg] * PAGE : p.cache_rows;
        return pg * PAGE < p.maxlen ? slot * p.maxlen + pg * PAGE : p.cache_rows;
      };
      int u = 0;
      auto load_tile = [&](const CUtensorMap* map, int kt) {
        const int r0 = page_row(2 * kt), r1 = page_row(2 * kt + 1);
        for (int hf = 0; hf < NU; ++hf, ++u) {
          const int st = u % RING;
          if (u >= RING && !mbar_wait(&u_empty[st], (u / RING - 1) & 1, p.err, 201)) return false;
          mbar_expect_tx(&u_full[st], 2 * SUB);
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            unsigned char* dst = smem + S::R0 + (st * 2 + c) * SUB;
            tma_load_4d(dst, map, &u_full[st], (hf * 2 + c) * 64, hk, r0, 0);
            tma_load_4d(dst + SUB / 2, map, &u_full[st], (hf * 2 + c) * 64, hk, r1, 0);
          }
        }
        return true;
      };
      bool ok = load_tile(&tmK, t0);
      for (int i = 1; ok && i < n; ++i) ok = load_tile(&tmK, t0 + i) && load_tile(&tmV, t0 + i - 1);
      if (ok) ok = load_tile(&tmV, t0 + n - 1);
      // the last units must have landed before the CTA can retire
      for (int v = (u > RING ? u - RING : 0); ok && v < u; ++v) mbar_wait(&u_full[v % RING], (v / RING) & 1, p.err, 202);
    }
  } else if (warp == 8) {
    // ---------------- MMA issuer ----------------
    if (lane == 0 && n > 0) {
      constexpr uint32_t idS = idesc_bf16_f32(BM, BN, 0, 0);
      constexpr uint32_t idPV = idesc_bf16_f32(BM, 128, 0, 1);
      const uint32_t sQ = smem_addr(smem + S::Q), sR = smem_addr(smem + S::R0);
      bool ok = mbar_wait(q_full, 0, p.err, 203);
      int u = 0;
      auto issue_s = [&](int i) {
        const int s = i & 1;
        // S_i goes over P_{i-2} in TMEM: PV_{i-2} must have read it
        if (i >= 2 && !mbar_wait(&pv_done[s], ((i - 2) >> 1) & 1, p.err, 211)) return false;
        for (int hf = 0; hf < NU; ++hf, ++u) {
          const int st = u % RING;
          if (!mbar_wait(&u_full[st], (u / RING) & 1, p.err, 204)) return false;
          tc_fence_after();
          const uint32_t base = sR + st * 2 * SUB;
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const int kg = hf * 8 + k;   // 16-column step over d
            umma_f16(tS[s], desc_sw128(sQ + (kg >> 2) * SUB + (kg & 3) * 32, 16, 1024),
                     desc_sw128(base + (k >> 2) * SUB + (k & 3) * 32, 16, 1024), idS, kg > 0 ? 1u : 0u);
          }
          umma_commit(&u_empty[st]);
        }
        umma_commit(&s_full[s]);
        return true;
      };
      auto issue_pv = [&](int j) {
        const uint32_t pcol = tS[j & 1];
        for (int hf = 0; hf < NU; ++hf, ++u) {
          const int st = u % RING;
          if (!mbar_wait(&u_full[st], (u / RING) & 1, p.err, 213)) return false;
          tc_fence_after();
          const uint32_t base = sR + st * 2 * SUB;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            // keys [16 kk, 16 kk + 16): P written by half kk / 4 at column 64 (kk / 4) + 8 (kk % 4)
            umma_f16_ts(tO + hf * 128, pcol + (kk >> 2) * 64 + (kk & 3) * 8, desc_sw128(base + kk * 2048, SUB, 1024),
                        idPV, (j > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&u_empty[st]);
        }
        umma_commit(&pv_done[j & 1]);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int i = 1; ok && i < n; ++i) {
        if (!(ok = issue_s(i))) break;
        if (!(ok = mbar_wait(&p_full[(i - 1) & 1], ((i - 1) >> 1) & 1, p.err, 205))) break;
        tc_fence_after();
        ok = issue_pv(i - 1);
      }
      if (ok && mbar_wait(&p_full[(n - 1) & 1], ((n - 1) >> 1) & 1, p.err, 206)) {
        tc_fence_after();
        issue_pv(n - 1);
      }
      umma_commit(drain);
      mbar_wait(drain, 0, p.err, 207);
    }
  } else {
    // ---------------- softmax / correction / epilogue (warps 0-7) ----------------
    const int half = warp >> 2;             // key columns [64 half, 64 half + 64) of each S tile
    const int r = (warp & 3) * 32 + lane;   // query row within the tile == TMEM lane
    const int ci = qt * p.rpt + r / p.G;    // canvas row of this query row
    const int h = hk * p.G + r % p.G;       // its query head
    // last visible key + 1: the whole canvas for MASK rows, keys up to the row itself for clean rows
    const int vis_end = ci >= p.n_clean ? kend : min(kend, pos + ci + 1);
    const int bar_id = 1 + (warp & 3);      // named barrier of warps (w, w + 4)
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    float* xch = reinterpret_cast<float*>(smem + S::XCH);
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int i = 0; i < n; ++i) {
      const int s = i & 1;
      const int lim = vis_end - ((t0 + i) * BN + half * 64);   // columns c < lim are visible
      if (ok) ok = mbar_wait(&s_full[s], (i >> 1) & 1, p.err, 208);
      float sv[64];
      float mx = -INFINITY;
      if (__all_sync(0xffffffffu, ok)) {
        tc_fence_after();
        uint32_t t[2][32];
        tmem_ld32(tS[s] + lane_off + half * 64, t[0]);
        tmem_ld32(tS[s] + lane_off + half * 64 + 32, t[1]);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int j = 0; j < 32; ++j) sv[c * 32 + j] = __uint_as_float(t[c][j]);
        if (lim < 64) {
#pragma unroll
          for (int c = 0; c < 64; ++c)
            if (c >= lim) sv[c] = -INFINITY;
        }
        float mxp[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) mxp[u] = sv[u];
#pragma unroll
        for (int c = 8; c < 64; ++c) mxp[c & 7] = fmaxf(mxp[c & 7], sv[c]);
        mx = fmaxf(fmaxf(fmaxf(mxp[0], mxp[1]), fmaxf(mxp[2], mxp[3])),
                   fmaxf(fmaxf(mxp[4], mxp[5]), fmaxf(mxp[6], mxp[7])));
      } else {
        ok = false;
      }
      // row max over both halves (the pair meets the barrier even after a timed-out wait)
      xch[half * BM + r] = mx;
      named_sync(bar_id, 64);
      mx = fmaxf(mx, xch[(1 - half) * BM + r]);
      named_sync(bar_id, 64);
      const float mx_s = mx * p.scale_log2;
      const bool grow = mx_s > m_run + RESCALE_THRESHOLD || (m_run == -INFINITY && mx_s > -INFINITY);
      // O may be rescaled only after PV_{i-1} has completed; TMEM loads / stores are warp-collective,
      // so when any row of the warp rescales, every lane loads and stores its O columns (alpha = 1
      // for rows that keep their max)
      const bool resc = grow && i > 0 && m_run != -INFINITY;
      if (__any_sync(0xffffffffu, resc && ok)) {
        if (ok) ok = mbar_wait(&pv_done[(i - 1) & 1], ((i - 1) >> 1) & 1, p.err, 209);
        tc_fence_after();
        const float alpha = (resc && ok) ? exp2f(m_run - mx_s) : 1.f;
        l_run *= alpha;
#pragma unroll 1
        for (int c = 0; c < D / 64; ++c) {       // this half's D / 2 columns of the O row
          uint32_t t[32];
          const uint32_t col = tO + lane_off + half * (D / 2) + c * 32;
          tmem_ld32(col, t);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) t[j] = __float_as_uint(__uint_as_float(t[j]) * alpha);
          tmem_st32(col, t);
        }
        tmem_wait_st();
      }
      if (grow) m_run = mx_s;
      if (__all_sync(0xffffffffu, ok)) {
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
      } else {
        ok = false;
      }
      tc_fence_before();
      mbar_arrive(&p_full[i & 1]);
    }
    if (ok && n > 0) ok = mbar_wait(&pv_done[(n - 1) & 1], ((n - 1) >> 1) & 1, p.err, 210);
    xch[half * BM + r] = l_run;
    named_sync(bar_id, 64);
    const float l_tot = l_run + xch[(1 - half) * BM + r];
    const bool row_ok = ci < p.blk;
    const bool have = __all_sync(0xffffffffu, ok) && n > 0;   // warp-uniform: TMEM loads are collective
    if (p.nsplit == 1) {
      bf16* dst = p.out + ((int64_t)(b * p.blk + ci) * p.Hq + h) * D + half * (D / 2);
      if (have) {
        tc_fence_after();
        const float inv = l_tot > 0.f ? 1.f / l_tot : 0.f;
#pragma unroll 1
        for (int c = 0; c < D / 64; ++c) {
          uint32_t t[32];
          tmem_ld32(tO + lane_off + half * (D / 2) + c * 32, t);
          tmem_wait_ld();
          if (row_ok) {
#pragma unroll
            for (int j8 = 0; j8 < 4; ++j8) {
              float f[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) f[j] = __uint_as_float(t[j8 * 8 + j]) * inv;
              store8(dst + c * 32 + j8 * 8, f);
            }
          }
        }
      }
    } else {
      const int64_t ri = (((int64_t)b * p.nsplit + split) * p.Hq + h) * p.blk + ci;
      if (have) {
        tc_fence_after();
        float* dst = p.po + ri * D + half * (D / 2);
#pragma unroll 1
        for (int c = 0; c < D / 64; ++c) {
          uint32_t t[32];
          tmem_ld32(tO + lane_off + half * (D / 2) + c * 32, t);
          tmem_wait_ld();
          if (row_ok) {
#pragma unroll
            for (int j4 = 0; j4 < 8; ++j4)
              *reinterpret_cast<float4*>(dst + c * 32 + j4 * 4) =
                  make_float4(__uint_as_float(t[j4 * 4]), __uint_as_float(t[j4 * 4 + 1]),
                              __uint_as_float(t[j4 * 4 + 2]), __uint_as_float(t[j4 * 4 + 3]));
          }
        }
      }
      if (row_ok && half == 0 && valid) {
        p.pm[ri] = (have && l_tot > 0.f) ? m_run : -INFINITY;
        p.pl[ri] = have ? l_tot : 0.f;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

}  // namespace canvas100

// q [B * blk, Hq, D] contiguous bf16; cache [rows, Hkv, D] as a 4-D map {D, Hkv, rows, 1}, boxes of
// 64 columns x 1 head x `rows_box` rows x 1.
static bool canvas_map(CUtensorMap* m, const void* base, int H, int D, int64_t rows, int box_h, int box_rows) {
  auto fn = attn100::encode_fn();
  if (!fn) return false;
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)rows, 1};
  cuuint64_t strides[3] = {(cuuint64_t)D * 2, (cuuint64_t)H * D * 2, (cuuint64_t)rows * H * D * 2};
  cuuint32_t box[4] = {64, (cuuint32_t)box_h, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

namespace canvas100 {
// Key splits: enough CTAs for two waves of one CTA per SM, but at least four key tiles per split.
static void plan(int B, int blk, int Hq, int Hkv, int max_keys, int& nqt, int& nsplit, int& tps) {
  static int sms = 0;
  if (sms == 0) {
    int dev = 0, n = 148;
    if (cudaGetDevice(&dev) == cudaSuccess && cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess)
      sms = n;
    else
      sms = 148;
  }
  const int rpt = BM / (Hq / Hkv);
  nqt = (blk + rpt - 1) / rpt;
  const int ctas = nqt * Hkv * B;
  const int tiles = std::max(1, (max_keys + BN - 1) / BN);
  nsplit = std::max(1, std::min((2 * sms + ctas - 1) / ctas, tiles / 4));
  tps = (tiles + nsplit - 1) / nsplit;
  nsplit = (tiles + tps - 1) / tps;
}
}  // namespace canvas100

int64_t canvas_tc_work_floats(int B, int blk, int Hq, int Hkv, int D, int max_keys) {
  int nqt, nsplit, tps;
  canvas100::plan(B, blk, Hq, Hkv, max_keys, nqt, nsplit, tps);
  const int64_t rows = (int64_t)B * nsplit * Hq * blk;
  return nsplit > 1 ? rows * D + 2 * rows : 0;
}

int canvas_attention_tc(const bf16* q, const bf16* kc, const bf16* vc, int64_t cache_rows, int n_slots,
                        const int* slot, const int* pos, bf16* out, float* work, int B, int blk, int n_clean, int Hq,
                        int Hkv, int D, int maxlen, int max_keys, float scale, int* err, cudaStream_t s,
                        const int* ptab, int maxpages) {
  using namespace canvas100;
  if (D != 128 && D != 256) return -1;
  const int G = Hq / Hkv;
  if (G * Hkv != Hq || G > BM || (BM % G) != 0) return -1;
  if (cache_rows >= INT_MAX || (int64_t)B * blk >= INT_MAX || max_keys > maxlen) return -1;
  if (((uintptr_t)q | (uintptr_t)kc | (uintptr_t)vc | (uintptr_t)out) & 15u) return -1;
  Params p;
  p.slot = slot; p.pos = pos; p.ptab = ptab; p.out = out; p.err = err;
  p.maxpages = maxpages; p.maxlen = maxlen; p.cache_rows = (int)cache_rows; p.n_slots = n_slots;
  p.blk = blk; p.n_clean = n_clean; p.Hq = Hq; p.G = G; p.rpt = BM / G;
  p.scale_log2 = scale * 1.44269504088896340736f;
  plan(B, blk, Hq, Hkv, max_keys, p.nqt, p.nsplit, p.tps);
  const int64_t rows = (int64_t)B * p.nsplit * Hq * blk;
  if (p.nsplit > 1 && work == nullptr) return -1;
  p.po = work; p.pm = p.nsplit > 1 ? work + rows * D : nullptr; p.pl = p.nsplit > 1 ? p.pm + rows : nullptr;

  CUtensorMap mq, mk, mv;
  if (!canvas_map(&mq, q, Hq, D, (int64_t)B * blk, G, BM / G)) return -2;
  if (!canvas_map(&mk, kc, Hkv, D, cache_rows, 1, PAGE)) return -3;
  if (!canvas_map(&mv, vc, Hkv, D, cache_rows, 1, PAGE)) return -4;
  const dim3 grid(p.nsplit, p.nqt * Hkv, B);
  if (D == 128) {
    constexpr int smem = Smem<128>::TOTAL + 1024;
    static bool init = false;
    if (!init) { cudaFuncSetAttribute(canvas_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem); init = true; }
    canvas_kernel<128><<<grid, NTH, smem, s>>>(mq, mk, mv, p);
  } else {
    constexpr int smem = Smem<256>::TOTAL + 1024;
    static bool init = false;
    if (!init) { cudaFuncSetAttribute(canvas_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem); init = true; }
    canvas_kernel<256><<<grid, NTH, smem, s>>>(mq, mk, mv, p);
  }
  if (p.nsplit > 1) canvas_combine(p.po, p.pm, p.pl, out, B, p.nsplit, Hq, blk, D, s);
  return cudaGetLastError() == cudaSuccess ? 0 : -5;
}

}  // namespace trida
