// Block-diffusion attention on the 5th-generation tensor cores (tcgen05 + TMEM): forward and backward.
//
// Forward.  CTA = one 128-row query tile of one head.  Warp roles (320 threads):
//   warps 0-7  softmax, two warpgroups splitting every row: thread (half, r) owns columns
//              [64 half, 64 half + 64) of query row r == TMEM lane r (warps w and w + 4 share a
//              TMEM lane quarter), so two warps per SM sub-partition hide each other's exp /
//              max / pack latencies.  At the start they copy their half of Q row r from the TMA
//              tile into TMEM (the A operand of every S MMA).  Per key tile each reads its half S
//              row with tcgen05.ld, applies the block-diffusion rule on PARTIAL tiles, exchanges
//              its half-row max with its partner through shared memory (named barrier per warp
//              pair), keeps the running max / sum, rescales its half of the O row in TMEM only when
//              the max grows by more than 2^16, and writes its half P row as bf16 pairs over its
//              own S columns in TMEM (the A operand of the PV MMA).  Control flow is identical in
//              both halves (a timed-out wait skips work but keeps meeting the pair barrier), so a
//              pair can never split.
//   warp 8     MMA issuer (one thread): S_i = Q K_i^T into one of two TMEM S buffers (after PV_{i-2},
//              which read P_{i-2} from the same columns, has completed), then O += P_{i-1} V_{i-1};
//              only the K / V tiles are read from shared memory.  Completion is signalled with
//              tcgen05.commit on mbarriers.
//   warp 9     TMA producer (one thread): Q once, K and V tiles into rings of their own (plain
//              per-CTA tensor loads, each CTA fetching its own tiles).
// TMEM columns: S0 [0,128), S1 [128,256), O [256, 256+D), Q [256+D, 256+D+D/2).  O leaves through
// the idle Q tile by TMA tensor stores.  The list of non-empty 128-key tiles (and whether each is
// FULL or PARTIAL) comes from the same exact classification pass as the other attention kernels.
// The backward is described above its kernel.  Every mbarrier wait is bounded; a timeout records
// an error code in a device word that the host checks, and the CTA still releases its TMEM.
#include <cudaTypedefs.h>

#include "common.cuh"
#include "ops.h"
#include "sm100_common.cuh"
#include "bd_attention_sm100.cuh"

#include <climits>

namespace trida {
namespace attn100 {

using namespace sm100;

constexpr int BM = 128, BN = 128;
constexpr int NTHREADS = 320;        // backward: 8 softmax-gradient warps + MMA warp + TMA warp
constexpr int FWD_THREADS = 320;     // forward: 8 softmax warps + MMA warp + TMA warp


struct Params {
  bf16* o;
  int64_t o_tok, o_b;
  float* lse;          // [B, Hq, T]
  const int4* meta;    // [B, T]
  const int16_t* list; // [B, nq128, nk128] entries kt | cls << 14
  const int* cnt;      // [B, nq128]
  const uint4* tmask;  // [B, nq128, nk128, 128] row bit-masks of PARTIAL tiles (bit c = key c allowed)
  int* err;
  long long* dbg;      // optional timeline: [cta][64 events] clock64 stamps (CTAs 0..7 only)
  int T, Hq, group, nk, flags;
  float scale_log2;
};

#define DBG_STAMP(slot)                                                                           \
  do {                                                                                            \
    if (p.dbg && cta_id < 8 && (slot) < 64) p.dbg[cta_id * 64 + (slot)] = clock64();              \
  } while (0)

template <int D>
struct Smem {
  static constexpr int SUB = BM * 128;                 // one [128 rows][64 bf16] swizzled sub-tile
  static constexpr int Q = 0;
  static constexpr int K0 = Q + (D / 64) * SUB;
  static constexpr int V0 = K0 + 2 * (D / 64) * SUB;
  static constexpr int XCH = V0 + 2 * (D / 64) * SUB;  // float[2 halves][128 rows]: half-row max / sum exchange
  static constexpr int BAR = XCH + 2 * 128 * 4;
  static constexpr int TOTAL = BAR + 256;
};



template <int D>
__global__ void __launch_bounds__(FWD_THREADS, 1)
    fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
               const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO, const Params p) {
  using S = Smem<D>;
  extern __shared__ unsigned char smem_raw[];
  // Align by pointer arithmetic on the __shared__ array (not an integer round-trip) so the compiler
  // keeps the shared address space and emits LDS/STS instead of generic loads/stores.
  unsigned char* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::BAR);
  // K and V have rings of their own: a K slot is free once its S MMA has run, a V slot once its PV
  // MMA has, so K_{i+1} streams in while the softmax of tile i runs instead of after PV_{i-1}.
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;     // [2]
  uint64_t* k_empty = bars + 3;    // [2]
  uint64_t* s_full = bars + 5;     // [2]
  uint64_t* p_full = bars + 7;
  uint64_t* pv_done = bars + 8;    // [2]: PV_j completes pv_done[j & 1] (completion number j >> 1)
  uint64_t* drain = bars + 10;
  uint64_t* v_full = bars + 11;    // [2]
  uint64_t* v_empty = bars + 13;   // [2]
  uint64_t* q_tmem = bars + 15;    // the softmax warps have copied Q into TMEM
  // p_full[0] = bars + 7, p_full[1] = bars + 16: P_i written completes p_full[i & 1] (S_{i+1} is
  // issued before PV_i, so a softmax warp can finish tile i+1 while another is still on tile i; one
  // barrier per parity keeps their arrivals apart)
  uint64_t* p_full1 = bars + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 17);

  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int hk = h / p.group;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nq = gridDim.x;
  const int lidx = b * nq + qt;
  const int n = p.cnt[lidx];
  const int16_t* list = p.list + (int64_t)lidx * p.nk;
  const int cta_id = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);

  if (threadIdx.x == 0) {
    DBG_STAMP(0);
    mbar_init(q_full, 1);
    for (int j = 0; j < 2; ++j) {
      mbar_init(&k_full[j], 1);
      mbar_init(&k_empty[j], 1);
      mbar_init(&v_full[j], 1);
      mbar_init(&v_empty[j], 1);
    }
    mbar_init(&s_full[0], 1);
    mbar_init(&s_full[1], 1);
    mbar_init(p_full, 2 * BM);
    mbar_init(p_full1, 2 * BM);
    mbar_init(q_tmem, 2 * BM);
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
  const uint32_t tQ = tmem + 256 + D;     // Q as the A operand: D / 2 columns of bf16 pairs

  if (warp == 9) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      mbar_expect_tx(q_full, (D / 64) * S::SUB);
#pragma unroll
      for (int c = 0; c < D / 64; ++c) tma_load_4d(smem + S::Q + c * S::SUB, &tmQ, q_full, c * 64, h, qt * BM, b);
      bool ok = true;
      for (int i = 0; ok && i < n; ++i) {
        const int s = i & 1;
        const int kt = list[i] & 0x3fff;
        if (i >= 2 && !(ok = mbar_wait(&k_empty[s], ((i - 2) >> 1) & 1, p.err, 1))) break;
        mbar_expect_tx(&k_full[s], (D / 64) * S::SUB);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_load_4d(smem + S::K0 + (s * (D / 64) + c) * S::SUB, &tmK, &k_full[s], c * 64, hk, kt * BN, b);
        if (i >= 2 && !(ok = mbar_wait(&v_empty[s], ((i - 2) >> 1) & 1, p.err, 12))) break;
        mbar_expect_tx(&v_full[s], (D / 64) * S::SUB);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_load_4d(smem + S::V0 + (s * (D / 64) + c) * S::SUB, &tmV, &v_full[s], c * 64, hk, kt * BN, b);
      }
      // drain: the last (up to two) loads must have landed before the CTA can retire
      for (int i = (n > 2 ? n - 2 : 0); ok && i < n; ++i) {
        mbar_wait(&k_full[i & 1], (i >> 1) & 1, p.err, 2);
        mbar_wait(&v_full[i & 1], (i >> 1) & 1, p.err, 2);
      }
    }
  } else if (warp == 8) {
    // ---------------- MMA issuer ----------------
    // A operands come from TMEM (Q copied there once by the softmax warps, P_i written over S_i),
    // so each MMA reads only its B tile (K_i or V_i) from shared memory.
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16_f32(BM, BN, 0, 0);
      constexpr uint32_t idPV = idesc_bf16_f32(BM, D, 0, 1);
      const uint32_t sK = smem_addr(smem + S::K0), sV = smem_addr(smem + S::V0);
      bool ok = mbar_wait(q_tmem, 0, p.err, 3);
      DBG_STAMP(1);
      auto issue_pv = [&](int j) {
        if (!mbar_wait(&v_full[j & 1], (j >> 1) & 1, p.err, 13)) return false;
        tc_fence_after();
        const uint32_t vbase = sV + (j & 1) * (D / 64) * S::SUB;
        const uint32_t pcol = tS[j & 1];
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          // keys [16 kk, 16 kk + 16): written by half kk / 4 at column 64 (kk / 4) + 8 (kk % 4)
          const uint64_t bd = desc_sw128(vbase + kk * 2048, S::SUB, 1024);
          umma_f16_ts(tO, pcol + (kk >> 2) * 64 + (kk & 3) * 8, bd, idPV, (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&pv_done[j & 1]);
        umma_commit(&v_empty[j & 1]);
        return true;
      };
      tc_fence_after();
      for (int i = 0; ok && i < n; ++i) {
        const int s = i & 1;
        if (!(ok = mbar_wait(&k_full[s], (i >> 1) & 1, p.err, 4))) break;
        // S_i goes over P_{i-2} in TMEM: PV_{i-2} must have read it
        if (i >= 2 && !(ok = mbar_wait(&pv_done[s], ((i - 2) >> 1) & 1, p.err, 11))) break;
        if (i < 6) DBG_STAMP(2 + 4 * i);
        tc_fence_after();
        const uint32_t kbase = sK + s * (D / 64) * S::SUB;
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint64_t bd = desc_sw128(kbase + (k >> 2) * S::SUB + (k & 3) * 32, 16, 1024);
          umma_f16_ts(tS[s], tQ + k * 8, bd, idS, k > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[s]);
        umma_commit(&k_empty[s]);
        if (i < 6) DBG_STAMP(3 + 4 * i);
        if (i > 0) {
          if (!(ok = mbar_wait(((i - 1) & 1) ? p_full1 : p_full, ((i - 1) >> 1) & 1, p.err, 5))) break;
          if (i < 6) DBG_STAMP(4 + 4 * i);
          tc_fence_after();
          if (!(ok = issue_pv(i - 1))) break;
        }
      }
      if (ok && n > 0 && mbar_wait(((n - 1) & 1) ? p_full1 : p_full, ((n - 1) >> 1) & 1, p.err, 6)) {
        tc_fence_after();
        issue_pv(n - 1);
      }
      // every MMA issued by this thread has completed once `drain` flips
      umma_commit(drain);
      mbar_wait(drain, 0, p.err, 7);
    }
  } else {
    // ---------------- softmax / correction / epilogue (warps 0-7) ----------------
    const int half = warp >> 2;             // columns [64 half, 64 half + 64) of the tile
    const int r = (warp & 3) * 32 + lane;   // query row within the tile == TMEM lane
    const int row = qt * BM + r;
    const int bar_id = 1 + (warp & 3);      // named barrier of warps (w, w + 4)
    const int4 mq = row < p.T ? p.meta[(int64_t)b * p.T + row] : make_int4(INT_MAX, INT_MAX, -3, SEG_PAD);
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    float* xch = reinterpret_cast<float*>(smem + S::XCH);
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    {  // copy this thread's half of Q row r from the TMA tile (128B-swizzled) into TMEM
      ok = mbar_wait(q_full, 0, p.err, 14);
      if (ok) {
        constexpr int NW = D / 4;                       // 32-bit words (bf16 pairs) per half row
        uint32_t w[NW];
#pragma unroll
        for (int u = 0; u < D / 16; ++u) {
          const int e = half * (D / 2) + u * 8;
          const uint4 v = *reinterpret_cast<const uint4*>(smem + S::Q + (e >> 6) * S::SUB + r * 128 +
                                                          ((((e & 63) >> 3) ^ (r & 7)) << 4));
          w[4 * u] = v.x; w[4 * u + 1] = v.y; w[4 * u + 2] = v.z; w[4 * u + 3] = v.w;
        }
        if constexpr (D == 128) tmem_st32(tQ + lane_off + half * NW, w);
        else tmem_st16(tQ + lane_off + half * NW, w);
        tmem_wait_st();
      }
      tc_fence_before();
      mbar_arrive(q_tmem);
    }
    for (int i = 0; i < n; ++i) {
      const int s = i & 1;
      const int entry = list[i];
      const int kt = entry & 0x3fff;
      const bool partial = (entry >> 14) != CLS_FULL;
      uint32_t bits[2];
      if (partial) {
        const uint4 w = p.tmask[(((int64_t)b * nq + qt) * p.nk + kt) * BM + r];
        bits[0] = half ? w.z : w.x;
        bits[1] = half ? w.w : w.y;
      }
      if (ok) ok = mbar_wait(&s_full[s], (i >> 1) & 1, p.err, 8);
      if (threadIdx.x == 0 && i < 6) DBG_STAMP(30 + 5 * i);
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
      named_sync(bar_id, 64);                           // both read before the next tile's write
      if (threadIdx.x == 0 && i < 6) DBG_STAMP(31 + 5 * i);
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
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {            // this half's columns of the O row
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
      if (ok) {
        // P_i (bf16 pairs) overwrites this half's own S_i columns in TMEM: 32 columns starting at
        // column 64 half, the A operand of PV_i
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
      mbar_arrive((i & 1) ? p_full1 : p_full);
      if (threadIdx.x == 0 && i < 6) DBG_STAMP(33 + 5 * i);
    }
    if (ok && n > 0) ok = mbar_wait(&pv_done[(n - 1) & 1], ((n - 1) >> 1) & 1, p.err, 10);
    if (threadIdx.x == 0) DBG_STAMP(60);
    // row sum over both halves
    xch[half * BM + r] = l_run;
    named_sync(bar_id, 64);
    const float l_tot = l_run + xch[(1 - half) * BM + r];
    // epilogue: O / l staged as bf16 in the (now idle) Q tile in the swizzled layout of the O
    // tensor map, then written by TMA as whole 128-row sub-tiles (coalesced; rows past T clipped)
    unsigned char* sO = smem + S::Q;
    const bool store = ok && n > 0;
    if (store) {
      tc_fence_after();
      const float inv = l_tot > 0.f ? 1.f / l_tot : 0.f;
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        uint32_t t[32];
        tmem_ld32(tO + lane_off + half * (D / 2) + c * 32, t);
        tmem_wait_ld();
#pragma unroll
        for (int j8 = 0; j8 < 4; ++j8) {
          float f[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) f[j] = __uint_as_float(t[j8 * 8 + j]) * inv;
          const int col = half * (D / 2) + c * 32 + j8 * 8;
          store8(reinterpret_cast<bf16*>(sO + (col >> 6) * S::SUB + sw128_offset(r, col & 63)), f);
        }
      }
      if (half == 0 && row < p.T)
        p.lse[((int64_t)b * p.Hq + h) * p.T + row] =
            (m_run == -INFINITY) ? -INFINITY : (m_run + log2f(l_tot)) * 0.69314718055994530942f;
      fence_async_smem();
    }
    named_sync(5, 256);                                 // the whole O tile is staged
    if (threadIdx.x == 0 && store) {
      if (threadIdx.x == 0) DBG_STAMP(61);
#pragma unroll
      for (int c = 0; c < D / 64; ++c) tma_store_4d(&tmO, sO + c * S::SUB, c * 64, h, qt * BM, b);
      asm volatile("cp.async.bulk.commit_group;\n" ::: "memory");
      asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory");
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x == 0) DBG_STAMP(63);
  if (warp == 0) tmem_dealloc(tmem, 512);
}


template <int D>
static int launch(const AttnTensors& t, const Params& p, int nq, cudaStream_t s) {
  CUtensorMap mq, mk, mv, mo;
  if (!make_map(&mq, t.q, t.B, t.T, t.Hq, D, t.q_tok, t.q_b)) return -2;
  if (!make_map(&mk, t.k, t.B, t.T, t.Hkv, D, t.k_tok, t.k_b)) return -3;
  if (!make_map(&mv, t.v, t.B, t.T, t.Hkv, D, t.v_tok, t.v_b)) return -4;
  if (!make_map(&mo, t.o, t.B, t.T, t.Hq, D, t.o_tok, t.o_b)) return -5;
  const int smem = Smem<D>::TOTAL + 1024;
  static bool init = false;
  if (!init) {
    cudaFuncSetAttribute(fwd_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    init = true;
  }
  fwd_kernel<D><<<dim3(nq, t.Hq, t.B), FWD_THREADS, smem, s>>>(mq, mk, mv, mo, p);
  return 0;
}


// =================================================================================================
// Backward.  CTA = one 128-key tile of one query head; it walks the non-empty 128-query tiles of
// its key tile.  Per pair j (warps 0-7: thread (g, r) owns key row r == TMEM lane r and query
// columns [64 g, 64 g + 64)):
//   MMA1  S^T  = K Q_j^T          -> TMEM [0,128)        (A = K  K-major, B = Q  K-major)
//   MMA2  dP^T = V dO_j^T         -> TMEM [128,256)      (A = V  K-major, B = dO K-major)
//   softmax-gradient warps, 32 queries at a time: P^T = exp2(S^T*scale*log2e - LSE2[q]) (masked
//         on PARTIAL tiles), dS^T = P^T * (dP^T - Dsum[q]); both written as bf16 K-major rows to smem.
//   MMA3  dV  += P^T dO_j         -> TMEM [256,256+D)    (A = P^T K-major, B = dO MN-major)
//   MMA4  dK  += dS^T Q_j         -> TMEM [384,384+D)    (A = dS^T K-major, B = Q MN-major)
//   MMA5  dQ_j = dS K             -> TMEM [0,128) again  (A = dS MN-major, B = K MN-major)
//   the same warps stage dQ_j (x scale, fp32) in the idle P^T / dS^T buffers and one thread adds
//   it to the fp32 dQ accumulator with TMA tensor reductions; TMEM [0,128) is then free again.
// At the end dK (x scale) and dV are added the same way into fp32 per-KV-head accumulators (the
// GQA group's query heads are separate CTAs).  Warp 8 issues MMAs, warp 9 issues TMA loads.
// =================================================================================================
struct BwdParams {
  bf16 *dk, *dv;
  int64_t dk_tok, dk_b, dv_tok, dv_b;
  float* dq_acc;            // [B, T, Hq, D] fp32, pre-zeroed
  float *dk_acc, *dv_acc;   // [B, T, Hkv, D] fp32, pre-zeroed (partials of the group's query heads)
  const float *lse, *dsum;  // [B, Hq, T]
  const int4* meta;
  const int16_t* list;      // [B, nk128, nq128] entries qt | cls << 14
  const int* cnt;           // [B, nk128]
  const uint4* tmask_t;     // [B, nk128, nq128, 128] column bit-masks of PARTIAL tiles (bit q = query q allowed)
  int* err;
  long long* dbg;
  int T, Hq, group, nq, flags;
  float scale, scale_log2;
};

template <int D>
struct BwdSmem {
  // K, V once per CTA; Q_j / dO_j double-buffered so pair j+1's tiles load while pair j runs, and
  // once pair j's MMAs have run its slot stages dQ_j for the TMA reductions; dS^T (bf16, K-major
  // rows = keys) is the A operand of dK and dQ.  P^T lives in TMEM only.
  static constexpr int SUB = 128 * 128;
  static constexpr int T = (D / 64) * SUB;      // one [128 rows][D] bf16 tile
  static constexpr int K = 0;
  static constexpr int V = K + T;
  static constexpr int Q = V + T;               // [2] tiles
  static constexpr int DO = Q + 2 * T;          // [2] tiles
  static constexpr int DST = DO + 2 * T;
  static constexpr int LSE = DST + 2 * SUB;     // float[128]
  static constexpr int DS = LSE + 512;          // float[128]
  static constexpr int BAR = DS + 512;
  static constexpr int TOTAL = BAR + 256;
};


template <int D>
__global__ void __launch_bounds__(NTHREADS, 1)
    bwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
               const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
               const __grid_constant__ CUtensorMap tmDQ, const __grid_constant__ CUtensorMap tmDK,
               const __grid_constant__ CUtensorMap tmDV, const BwdParams p) {
  using S = BwdSmem<D>;
  extern __shared__ unsigned char smem_raw[];
  // Align by pointer arithmetic on the __shared__ array (not an integer round-trip) so the compiler
  // keeps the shared address space and emits LDS/STS instead of generic loads/stores.
  unsigned char* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::BAR);
  uint64_t* kv_full = bars + 0;
  uint64_t* q_full = bars + 1;    // [2]
  uint64_t* q_empty = bars + 3;   // [2]
  uint64_t* sp_full = bars + 5;
  uint64_t* p_full = bars + 6;
  uint64_t* dq_full = bars + 7;   // every MMA of the pair has completed (dQ_j is in TMEM)
  uint64_t* dq_free = bars + 8;   // the softmax warps have read dQ_j out of TMEM
  uint64_t* drain = bars + 9;
  uint64_t* slot_free = bars + 10; // [2]: the dQ reductions staged in a Q / dO slot have read it
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);
  float* sLSE = reinterpret_cast<float*>(smem + S::LSE);
  float* sDs = reinterpret_cast<float*>(smem + S::DS);

  // one CTA per (key tile, query head): the GQA group's heads are separate CTAs whose dK / dV
  // partials meet in fp32 accumulators (TMA reduce-add), so no CTA walks group x query tiles
  const int kt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int hk = h / p.group;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = gridDim.x;
  const int lidx = b * nk + kt;
  const int total = p.cnt[lidx];
  const int16_t* list = p.list + (int64_t)lidx * p.nq;
  // CTAs of neighbouring key tiles start their walk at different query tiles so their dQ
  // reductions land on different rows at any moment.
  const int rot = total > 0 ? (kt * 7 + h * 3) % total : 0;
  const int cta_id = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);

  if (threadIdx.x == 0) {
    DBG_STAMP(0);
    mbar_init(kv_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&slot_free[i], 1);
    }
    mbar_init(sp_full, 1);
    mbar_init(p_full, 256);
    mbar_init(dq_full, 1);
    mbar_init(dq_free, 256);
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // TMEM: S^T [0,128) then P^T (bf16 pairs, written over it); dP^T [128,256) then dQ_j; dV; dK
  const uint32_t tS = tmem, tDP = tmem + 128, tDV = tmem + 256, tDK = tmem + 256 + D;

  if (warp == 9) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      prefetch_tmap(&tmDO);
      mbar_expect_tx(kv_full, 2 * S::T);
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        tma_load_4d(smem + S::K + c * S::SUB, &tmK, kv_full, c * 64, hk, kt * 128, b);
        tma_load_4d(smem + S::V + c * S::SUB, &tmV, kv_full, c * 64, hk, kt * 128, b);
      }
      for (int j = 0; j < total; ++j) {
        const int s = j & 1;
        // slot s held pair j-2: its MMAs have run and the dQ_{j-2} reductions staged there have read it
        if (j >= 2 && !mbar_wait(&q_empty[s], ((j - 2) >> 1) & 1, p.err, 21)) break;
        if (j >= 2 && !mbar_wait(&slot_free[s], ((j - 2) >> 1) & 1, p.err, 31)) break;
        const int qt = list[(j + rot) % total] & 0x3fff;
        mbar_expect_tx(&q_full[s], 2 * S::T);
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          tma_load_4d(smem + S::Q + s * S::T + c * S::SUB, &tmQ, &q_full[s], c * 64, h, qt * 128, b);
          tma_load_4d(smem + S::DO + s * S::T + c * S::SUB, &tmDO, &q_full[s], c * 64, h, qt * 128, b);
        }
      }
      // the last (up to two) loads must have landed before the CTA can retire
      for (int j = (total > 2 ? total - 2 : 0); j < total; ++j) mbar_wait(&q_full[j & 1], (j >> 1) & 1, p.err, 22);
    }
  } else if (warp == 8) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idKK = idesc_bf16_f32(128, 128, 0, 0);   // S^T, dP^T
      constexpr uint32_t idKM = idesc_bf16_f32(128, D, 0, 1);     // dV (A from TMEM), dK (B MN-major)
      constexpr uint32_t idMM = idesc_bf16_f32(128, D, 1, 1);     // dQ (A and B MN-major)
      const uint32_t sK = smem_addr(smem + S::K), sV = smem_addr(smem + S::V), sQ0 = smem_addr(smem + S::Q),
                     sDO0 = smem_addr(smem + S::DO), sDST = smem_addr(smem + S::DST);
      bool ok = mbar_wait(kv_full, 0, p.err, 23);
      for (int j = 0; ok && j < total; ++j) {
        const int s = j & 1;
        const uint32_t sQ = sQ0 + s * S::T, sDO = sDO0 + s * S::T;
        if (!(ok = mbar_wait(&q_full[s], (j >> 1) & 1, p.err, 24))) break;
        // S^T_j goes over P^T_{j-1}: every MMA of pair j-1 (dV read P^T) has completed
        if (j > 0 && !(ok = mbar_wait(dq_full, (j - 1) & 1, p.err, 25))) break;
        if (j < 6) DBG_STAMP(10 + 3 * j);
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint32_t off = (k >> 2) * S::SUB + (k & 3) * 32;
          umma_f16(tS, desc_sw128(sK + off, 16, 1024), desc_sw128(sQ + off, 16, 1024), idKK, k > 0);
        }
        // dP^T_j goes over dQ_{j-1}: the softmax warps have read it out
        if (j > 0 && !(ok = mbar_wait(dq_free, (j - 1) & 1, p.err, 30))) break;
        if (j < 6) DBG_STAMP(11 + 3 * j);
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint32_t off = (k >> 2) * S::SUB + (k & 3) * 32;
          umma_f16(tDP, desc_sw128(sV + off, 16, 1024), desc_sw128(sDO + off, 16, 1024), idKK, k > 0);
        }
        umma_commit(sp_full);
        if (!(ok = mbar_wait(p_full, j & 1, p.err, 26))) break;
        if (j < 6) DBG_STAMP(12 + 3 * j);
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 128 / 16; ++kk) {
          // queries [16 kk, 16 kk + 16): P^T written by group kk / 4 at column 64 (kk / 4) + 8 (kk % 4)
          const uint32_t aoff = (kk >> 2) * S::SUB + (kk & 3) * 32;   // K-major 16-query step (dS^T)
          const uint32_t boff = kk * 2048;                            // MN-major 16-row step
          const uint32_t acc = (j > 0 || kk > 0) ? 1u : 0u;
          umma_f16_ts(tDV, tS + (kk >> 2) * 64 + (kk & 3) * 8, desc_sw128(sDO + boff, S::SUB, 1024), idKM, acc);
          umma_f16(tDK, desc_sw128(sDST + aoff, 16, 1024), desc_sw128(sQ + boff, S::SUB, 1024), idKM, acc);
        }
#pragma unroll
        for (int kk = 0; kk < 128 / 16; ++kk) {
          // A = dS (M = queries, K = keys): the dS^T rows (key-major) read as MN-major, 16 keys per step
          umma_f16(tDP, desc_sw128(sDST + kk * 2048, S::SUB, 1024), desc_sw128(sK + kk * 2048, S::SUB, 1024), idMM,
                   kk > 0);
        }
        umma_commit(dq_full);
        umma_commit(&q_empty[s]);
      }
      umma_commit(drain);
      mbar_wait(drain, 0, p.err, 27);
    }
  } else {
    // ---------------- warps 0-7: two warpgroups, g = threadIdx.x / 128 ----------------
    // Thread (g, r) owns key row r (TMEM lane r; warps w and w + 4 share a lane quarter) and the
    // query columns [64 g, 64 g + 64) of S^T / dP^T, so two warps per SM sub-partition overlap
    // each other's TMEM loads, exponentials and packing.  The dQ, dK and dV read-outs split their
    // D / 32 column chunks between the two groups the same way.
    const int r = threadIdx.x & 127, g = threadIdx.x >> 7;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    constexpr int CPG = D / 64;                 // 32-column read-out chunks per group
    unsigned char* sDST = smem + S::DST;
    bool ok = true;
    // Per-pair inputs (list entry, LSE / Dsum of the query row, PARTIAL-tile mask) are loaded one
    // pair ahead, during the softmax of the previous pair, so no global round trip sits between
    // two pairs.
    int e_next = total > 0 ? list[rot % total] : 0;
    float lse_next = -INFINITY, ds_next = 0.f;
    uint2 cm_next = make_uint2(0xffffffffu, 0xffffffffu);
    auto fetch = [&](int e) {
      const int qn = (e & 0x3fff) * 128 + r;
      if (g == 0) {
        const int64_t li = ((int64_t)b * p.Hq + h) * p.T + qn;
        lse_next = qn < p.T ? -p.lse[li] * 1.44269504088896340736f : -INFINITY;   // staged negated
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
      const int entry = e_next;
      const int qt = entry & 0x3fff;
      const uint2 cm = cm_next;
      if (g == 0) {  // this query tile's -LSE (log2 domain) and -Dsum
        sLSE[r] = lse_next;
        sDs[r] = ds_next;
      }
      if (j + 1 < total) e_next = list[(j + 1 + rot) % total];
      named_bar_sync(1, 256);
      if (threadIdx.x == 0 && j < 6) DBG_STAMP(40 + 4 * j);
      if (!(ok = mbar_wait(sp_full, j & 1, p.err, 28))) break;
      if (threadIdx.x == 0 && j < 6) DBG_STAMP(41 + 4 * j);
      tc_fence_after();
      if (j + 1 < total) fetch(e_next);
      // four 16-query sub-chunks of this group's 64 columns; the next sub-chunk's S^T / dP^T loads
      // are in flight while the current one is computed
      uint32_t sv[2][16], dv[2][16];
      tmem_ld16(tS + lane_off + g * 64, sv[0]);
      tmem_ld16(tDP + lane_off + g * 64, dv[0]);
#pragma unroll
      for (int sc = 0; sc < 4; ++sc) {
        const int cur = sc & 1;
        const int q0 = g * 64 + sc * 16;            // first query column of the sub-chunk
        tmem_wait_ld();
        if (sc < 3) {
          tmem_ld16(tS + lane_off + q0 + 16, sv[cur ^ 1]);
          tmem_ld16(tDP + lane_off + q0 + 16, dv[cur ^ 1]);
        }
        const uint32_t amask = ((sc < 2 ? cm.x : cm.y) >> ((sc & 1) * 16)) & 0xffffu;
        // two queries per packed fp32x2 step: x = S^T * scale_log2 - LSE2, P^T = exp2(x) (masked
        // on PARTIAL tiles), dS^T = P^T * (dP^T - Dsum); P^T and dS^T packed to bf16 pairs
        const uint64_t scale2 = f2pack(p.scale_log2, p.scale_log2);
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
        // P^T (bf16 pairs, the A operand of dV) over S^T columns [64 g + 8 sc, 64 g + 8 sc + 8),
        // whose values were loaded with sub-chunk sc / 2
        tmem_st8(tS + lane_off + g * 64 + sc * 8, pw);
#pragma unroll
        for (int t8 = 0; t8 < 2; ++t8) {
          const int col = q0 + t8 * 8;
          *reinterpret_cast<uint4*>(sDST + (col >> 6) * S::SUB + sw128_offset(r, col & 63)) =
              make_uint4(dw[t8 * 4], dw[t8 * 4 + 1], dw[t8 * 4 + 2], dw[t8 * 4 + 3]);
        }
      }
      tmem_wait_st();
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(p_full);
      if (threadIdx.x == 0 && j > 0) {   // pair j-1's dQ reductions have read their slot (this
        bulk_wait_read();                 // thread is idle until the MMAs of pair j complete)
        mbar_arrive(&slot_free[(j - 1) & 1]);
      }
      if (threadIdx.x == 0 && j < 6) DBG_STAMP(42 + 4 * j);
      if (!(ok = mbar_wait(dq_full, j & 1, p.err, 29))) break;
      if (threadIdx.x == 0 && j < 6) DBG_STAMP(43 + 4 * j);
      tc_fence_after();
      // dQ_j rows (lane r = query qt*128 + r): read this group's chunks, release TMEM for dP^T_{j+1},
      // then stage them (x scale, fp32, 128B-swizzled 16 KB chunks) in this pair's Q / dO slot,
      // idle now that its MMAs have run (pair j+1 is already in the other slot), and add them to the
      // fp32 accumulator with TMA tensor reductions that overlap pair j+1; the producer refills the
      // slot once they have read it (slot_free, signalled during pair j+1).
      {
        uint32_t t[CPG][32];
#pragma unroll
        for (int cc = 0; cc < CPG; ++cc) tmem_ld32(tDP + lane_off + (g * CPG + cc) * 32, t[cc]);
        tmem_wait_ld();
        tc_fence_before();
        mbar_arrive(dq_free);
        const int sl = j & 1;
#pragma unroll
        for (int cc = 0; cc < CPG; ++cc) {
          const int c = g * CPG + cc;       // chunks [0, D/64) in the Q tile, the rest in the dO tile
          unsigned char* sc = c < D / 64 ? smem + S::Q + sl * S::T + c * S::SUB
                                         : smem + S::DO + sl * S::T + (c - D / 64) * S::SUB;
#pragma unroll
          for (int u = 0; u < 8; ++u)
            *reinterpret_cast<float4*>(sc + r * 128 + ((u ^ (r & 7)) << 4)) =
                make_float4(__uint_as_float(t[cc][u * 4]) * p.scale, __uint_as_float(t[cc][u * 4 + 1]) * p.scale,
                            __uint_as_float(t[cc][u * 4 + 2]) * p.scale, __uint_as_float(t[cc][u * 4 + 3]) * p.scale);
        }
        fence_async_smem();
        named_bar_sync(1, 256);
        if (threadIdx.x == 0) {
          for (int c = 0; c < D / 32; ++c) {
            const unsigned char* sc = c < D / 64 ? smem + S::Q + sl * S::T + c * S::SUB
                                                 : smem + S::DO + sl * S::T + (c - D / 64) * S::SUB;
            tma_reduce_add_4d(&tmDQ, sc, c * 32, h, qt * 128, b);
          }
          bulk_commit();
        }
      }
    }
    if (threadIdx.x == 0) DBG_STAMP(62);
    if (threadIdx.x == 0) {
      bulk_wait_read();                         // the last dQ reductions have read their slot
      if (ok && total > 0) mbar_arrive(&slot_free[(total - 1) & 1]);
    }
    named_bar_sync(1, 256);
    if (ok && total > 0) {
      // dK (x scale) and dV partials of this query head, staged in the idle Q / dO tiles and added
      // by TMA into the fp32 accumulators shared by the group's heads (rows past T are clipped)
      unsigned char* stage = smem + S::Q;
#pragma unroll 1
      for (int which = 0; which < 2; ++which) {
        const uint32_t src = which == 0 ? tDK : tDV;
        const float mul = which == 0 ? p.scale : 1.f;
#pragma unroll 1
        for (int cc = 0; cc < CPG; ++cc) {
          const int c = g * CPG + cc;
          uint32_t t[32];
          tmem_ld32(src + lane_off + c * 32, t);
          tmem_wait_ld();
          unsigned char* sc = stage + c * (128 * 128);
#pragma unroll
          for (int u = 0; u < 8; ++u)
            *reinterpret_cast<float4*>(sc + r * 128 + ((u ^ (r & 7)) << 4)) =
                make_float4(__uint_as_float(t[u * 4]) * mul, __uint_as_float(t[u * 4 + 1]) * mul,
                            __uint_as_float(t[u * 4 + 2]) * mul, __uint_as_float(t[u * 4 + 3]) * mul);
        }
        fence_async_smem();
        named_bar_sync(1, 256);
        if (threadIdx.x == 0) {
#pragma unroll 1
          for (int c = 0; c < D / 32; ++c)
            tma_reduce_add_4d(which == 0 ? &tmDK : &tmDV, stage + c * (128 * 128), c * 32, hk, kt * 128, b);
          bulk_commit();
          bulk_wait_read();
        }
        named_bar_sync(1, 256);
      }
    }
    if (threadIdx.x == 0) bulk_wait_all();    // every reduction issued by this CTA has completed
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x == 0) DBG_STAMP(63);
  if (warp == 0) tmem_dealloc(tmem, 512);
}


template <int D>
static int launch_bwd(const AttnTensors& t, const bf16* dout, int64_t do_tok, int64_t do_b, const BwdParams& p,
                      int nk, cudaStream_t s) {
  CUtensorMap mq, mk, mv, mdo, mdq, mdk, mdv;
  if (!make_map_f32(&mdq, p.dq_acc, t.B, t.T, t.Hq, D)) return -6;
  if (!make_map_f32(&mdk, p.dk_acc, t.B, t.T, t.Hkv, D)) return -7;
  if (!make_map_f32(&mdv, p.dv_acc, t.B, t.T, t.Hkv, D)) return -8;
  if (!make_map(&mq, t.q, t.B, t.T, t.Hq, D, t.q_tok, t.q_b)) return -2;
  if (!make_map(&mk, t.k, t.B, t.T, t.Hkv, D, t.k_tok, t.k_b)) return -3;
  if (!make_map(&mv, t.v, t.B, t.T, t.Hkv, D, t.v_tok, t.v_b)) return -4;
  if (!make_map(&mdo, dout, t.B, t.T, t.Hq, D, do_tok, do_b)) return -5;
  const int smem = BwdSmem<D>::TOTAL + 1024;
  static bool init = false;
  if (!init) {
    cudaFuncSetAttribute(bwd_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    init = true;
  }
  bwd_kernel<D><<<dim3(nk, t.Hq, t.B), NTHREADS, smem, s>>>(mq, mk, mv, mdo, mdq, mdk, mdv, p);
  return 0;
}

// Bit masks of every PARTIAL 128x128 tile, evaluated once per forward (shared by all heads,
// layers and both passes): row masks (thread = query row, bit = key) for the forward and column
// masks (thread = key row, bit = query) for the backward.
__global__ void tile_masks_kernel(const int4* __restrict__ meta, const uint8_t* __restrict__ cls, int B, int T,
                                  int nt, int n128, int flags, uint4* __restrict__ rowmask,
                                  uint4* __restrict__ colmask) {
  __shared__ int4 mq[128], mk[128];
  const int kt = blockIdx.x, qt = blockIdx.y, b = blockIdx.z;
  int any = 0, all = 1;
  for (int dq = 0; dq < 2; ++dq)
    for (int dk = 0; dk < 2; ++dk) {
      const int qi = 2 * qt + dq, ki = 2 * kt + dk;
      const int v = (qi < nt && ki < nt) ? cls[((int64_t)b * nt + qi) * nt + ki] : 0;
      any |= v != 0;
      all &= (v == 1) && ki < nt;
    }
  if (!any || all) return;   // EMPTY or FULL tile: no mask needed (a uniform branch)
  const int r = threadIdx.x;
  const int qrow = qt * 128 + r, krow = kt * 128 + r;
  mq[r] = qrow < T ? meta[(int64_t)b * T + qrow] : make_int4(INT_MAX, INT_MAX, -7, SEG_PAD);
  mk[r] = krow < T ? meta[(int64_t)b * T + krow] : make_int4(INT_MAX, INT_MAX, -8, SEG_PAD);
  __syncthreads();
  uint32_t rw[4] = {0, 0, 0, 0}, cw[4] = {0, 0, 0, 0};
  for (int c = 0; c < 128; ++c) {
    const int kj = kt * 128 + c, qi = qt * 128 + c;
    const bool ra = qrow < T && kj < T && allowed(mq[r], mk[c], qrow == kj, flags);
    const bool ca = krow < T && qi < T && allowed(mq[c], mk[r], qi == krow, flags);
    rw[c >> 5] |= (uint32_t)ra << (c & 31);
    cw[c >> 5] |= (uint32_t)ca << (c & 31);
  }
  rowmask[(((int64_t)b * n128 + qt) * n128 + kt) * 128 + r] = make_uint4(rw[0], rw[1], rw[2], rw[3]);
  colmask[(((int64_t)b * n128 + kt) * n128 + qt) * 128 + r] = make_uint4(cw[0], cw[1], cw[2], cw[3]);
}

// Lists at 128x128 granularity from the exact 64x64 classes.  transpose = 0: per query tile, the
// key tiles (forward); transpose = 1: per key tile, the query tiles (backward).
__global__ void lists128_kernel(const uint8_t* __restrict__ cls, int B, int nt, int nq, int nk,
                                int16_t* __restrict__ list, int* __restrict__ cnt, int transpose) {
  const int tid = blockIdx.x * blockDim.x + threadIdx.x;
  if (tid >= B * nq) return;
  const int b = tid / nq, q = tid % nq;
  int c = 0;
  for (int k = 0; k < nk; ++k) {
    int any = 0, all = 1;
    for (int dq = 0; dq < 2; ++dq)
      for (int dk = 0; dk < 2; ++dk) {
        const int qi = transpose ? 2 * k + dq : 2 * q + dq, ki = transpose ? 2 * q + dk : 2 * k + dk;
        const int v = (qi < nt && ki < nt) ? cls[((int64_t)b * nt + qi) * nt + ki] : 0;
        any |= v != 0;
        all &= (v == 1) || qi >= nt;   // rows beyond T are never stored
        if (ki >= nt) all = 0;
      }
    if (!any) continue;
    list[(int64_t)tid * nk + c] = (int16_t)(k | ((all ? 1 : 2) << 14));
    ++c;
  }
  cnt[tid] = c;
}

}  // namespace attn100

int bd_attn_bwd_sm100(const AttnTensors& t, const bf16* dout, int64_t do_tok, int64_t do_b, const float* dsum,
                      float* dq_acc, float* dk_acc, float* dv_acc, bf16* dk, int64_t dk_tok, int64_t dk_b, bf16* dv,
                      int64_t dv_tok, int64_t dv_b, const int4* meta, const int16_t* list128t, const int* cnt128t,
                      const uint4* colmask, int flags, float scale, int* err, cudaStream_t s, long long* dbg) {
  attn100::BwdParams p;
  p.dk_acc = dk_acc; p.dv_acc = dv_acc;
  p.dbg = dbg;
  p.tmask_t = colmask;
  p.dk = dk; p.dv = dv; p.dk_tok = dk_tok; p.dk_b = dk_b; p.dv_tok = dv_tok; p.dv_b = dv_b;
  p.dq_acc = dq_acc; p.lse = t.lse; p.dsum = dsum; p.meta = meta; p.list = list128t; p.cnt = cnt128t; p.err = err;
  p.T = t.T; p.Hq = t.Hq; p.group = t.Hq / t.Hkv; p.nq = (t.T + 127) / 128; p.flags = flags;
  p.scale = scale; p.scale_log2 = scale * 1.44269504088896340736f;
  const int nk = (t.T + 127) / 128;
  switch (t.D) {
    case 64: return attn100::launch_bwd<64>(t, dout, do_tok, do_b, p, nk, s);
    case 128: return attn100::launch_bwd<128>(t, dout, do_tok, do_b, p, nk, s);
    default: return -1;
  }
}

void bd_attn_tile_masks(const int4* meta, const uint8_t* cls, int B, int T, int flags, uint4* rowmask, uint4* colmask,
                        cudaStream_t s) {
  const int nt = (T + 63) / 64, n128 = (T + 127) / 128;
  attn100::tile_masks_kernel<<<dim3(n128, n128, B), 128, 0, s>>>(meta, cls, B, T, nt, n128, flags, rowmask, colmask);
}

void bd_attn_lists128(const uint8_t* cls, int B, int T, int16_t* list, int* cnt, int transpose, cudaStream_t s) {
  const int nt = (T + 63) / 64, n128 = (T + 127) / 128;
  attn100::lists128_kernel<<<ceil_div(B * n128, 128), 128, 0, s>>>(cls, B, nt, n128, n128, list, cnt, transpose);
}

int bd_attn_fwd_sm100(const AttnTensors& t, const int4* meta, const int16_t* list128, const int* cnt128,
                      const uint4* rowmask, int flags, float scale, int* err, cudaStream_t s, long long* dbg) {
  attn100::Params p;
  p.dbg = dbg;
  p.tmask = rowmask;
  p.o = t.o; p.o_tok = t.o_tok; p.o_b = t.o_b; p.lse = t.lse; p.meta = meta;
  p.list = list128; p.cnt = cnt128; p.err = err;
  p.T = t.T; p.Hq = t.Hq; p.group = t.Hq / t.Hkv; p.nk = (t.T + 127) / 128; p.flags = flags;
  p.scale_log2 = scale * 1.44269504088896340736f;
  const int nq = (t.T + 127) / 128;
  switch (t.D) {
    case 64: return attn100::launch<64>(t, p, nq, s);
    case 128: return attn100::launch<128>(t, p, nq, s);
    case 256: return bd_attn_fwd_d256(t, list128, cnt128, rowmask, meta, flags, scale, err, s);
    default: return -1;
  }
}

}  // namespace trida
