// Chunked (WY) gated-delta rule on the 5th-generation tensor cores (sm_100a).
//
// The math is the chunk decomposition stated in trida_stack_b200/ops/gdn_chunked.py (reference
// semantics: train/models/hybrid.py:137-212 causal rule with document resets, :215-324 two-stream
// block-diffusion form).  Per chunk of C tokens with entering state S0 [dk, dv]:
//     A = strict-lower(beta_t k_t.k_s e^{G_t - G_s}),  T = (I + A)^-1
//     W = T diag(beta carry e^G) K,  U~ = T diag(beta) V,  U = U~ - W S0
//     O = diag(carry e^{Gr}) Q S0 + P U,  P_ts = q_t.k_s e^{Gr_t - G_s} (s <= r(t), same segment)
//     S1 = carry_last e^{G_last} S0 + K~^T U
//
// Work is organised in 128-row tiles (128 / C chunks each; C = 64 for the causal layout, C = the
// diffusion block for the two-stream layout, so every block start is a chunk start).  Every
// operand is a 128 x 128 bf16 tile in shared memory, stored row-major as two [128][64] 128-byte
// swizzled halves (the layout TMA writes with a 64-element box), and every product is one
// M = 128 tcgen05.mma chain with its accumulator in TMEM.  The same stored tile X[r][c] serves as
//     A (M = r, K = c) or B (N = r, K = c)  through a K-major descriptor,
//     A (M = c, K = r) or B (N = c, K = r)  through an MN-major descriptor,
// so transposes cost nothing; products whose result must be transposed are simply computed in
// the transposed orientation (e.g. U^T = U~^T - S0^T W^T with the value dimension on the TMEM
// lanes).  Threads own TMEM lanes = tile rows: thread r reads row r of an accumulator, applies the
// masks / decays / row scales in registers and writes the bf16 operand of the next product.
//
// Kernels (one launch each, per layer):
//   chunk_prep  : L2-normalised q (times scale) / k in bf16 for the MMAs, log-decay g and beta.
//   local (PREP): per clean tile: T, -W, U~ and K~ (state-free, fully parallel).
//   scan        : per (row, value head), sequential over the clean chunks: stores the chunk-start
//                 states (bf16) and U = U~ - W S (two MMAs per chunk, fp32 state in TMEM).
//   local (OUT) : per clean tile: O from Q, K, U and the chunk-start states.
//   local (NOISY): per noisy tile of the two-stream layout: everything above from the stored clean
//                 state at the block start (no scan: noisy blocks are independent).
// Every mbarrier wait is bounded (error word, never a hang); no TMA load uses cluster multicast.
#include "gdn_chunk.cuh"

namespace trida {
namespace gdnc {

using namespace trida::sm100;

// ---- local kernel ----------------------------------------------------------------------------------
struct LocalSmem {
  static constexpr int R0 = 0;                    // Q -> Qg -> O staging
  static constexpr int R1 = R0 + TILE;            // K -> Kb -> state buffer 0
  static constexpr int R2 = R1 + TILE;            // V -> Vb -> P
  static constexpr int R3 = R2 + TILE;            // T -> U^T (noisy) / U (out, TMA)
  static constexpr int R4 = R3 + TILE;            // A blocks (fp32) -> -W
  static constexpr int R5 = R4 + AF_BYTES;        // state buffer 1
  static constexpr int R5A = R5;
  static constexpr int META = R5A + TILE;
  static constexpr int BARS = META + Meta::BYTES;
  static constexpr int TOTAL = BARS + 64;
};

// Grid (tiles, Hv, B [* V for NOISY]).
template <int MODE, int C>
__global__ void __launch_bounds__(NT, 1) local_kernel(const __grid_constant__ CUtensorMap tm_qk,
                                                      const __grid_constant__ CUtensorMap tm_v,
                                                      const __grid_constant__ CUtensorMap tm_u,
                                                      const __grid_constant__ CUtensorMap tm_st, const Args a,
                                                      int v_col0) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  using S = LocalSmem;
  using WN = Win<C>;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + S::BARS);
  uint64_t* ld_bar = bars;          // TMA loads of Q / K / V (or U)
  uint64_t* mma_bar = bars + 1;     // tcgen05.commit
  uint64_t* st_bar = bars + 2;      // state loads (two buffers)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 4);
  const Meta m = carve_meta(sm + S::META);
  const int r = threadIdx.x;
  constexpr int NCK = TR / C;

  TileGeo t;
  t.hv = blockIdx.y;
  t.hk = t.hv / (a.Hv / a.Hk);
  if (MODE == NOISY) {
    t.b = blockIdx.z / a.V;
    t.stream = 1 + blockIdx.z % a.V;
  } else {
    t.b = blockIdx.z;
    t.stream = 0;
  }
  t.Ls = clean_len(a);
  t.p0 = blockIdx.x * TR;
  t.t0 = t.stream * a.L + t.p0;
  t.tok = (t.stream == 0) ? (a.mode == 0 || a.tok_clean) : a.tok_noisy;

  if (r == 0) {
    mbar_init(ld_bar, 1);
    mbar_init(mma_bar, 1);
    mbar_init(&st_bar[0], 1);
    mbar_init(&st_bar[1], 1);
    fence_barrier_init();
  }
  if (r < 32) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t acc0 = tmem, acc1 = tmem + 128, acc2 = tmem + 256, acc3 = tmem + 384;
  const uint32_t sbase = smem_addr(sm);
  uint32_t mph = 0;       // phases of mma_bar consumed so far
  bool ok = true;

  // ---- loads: Q, K and V (or U for OUT) -----------------------------------------------------------
  if (r == 0) {
    prefetch_tmap(&tm_qk);
    mbar_expect_tx(ld_bar, 3 * TILE);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      tma_load_4d(sm + S::R0 + h * SUB, &tm_qk, ld_bar, h * 64, 2 * t.hk, t.t0, t.b);
      tma_load_4d(sm + S::R1 + h * SUB, &tm_qk, ld_bar, h * 64, 2 * t.hk + 1, t.t0, t.b);
      if (MODE == OUT)
        tma_load_4d(sm + S::R3 + h * SUB, &tm_u, ld_bar, h * 64, t.hv, t.t0, t.b);
      else
        tma_load_4d(sm + S::R2 + h * SUB, &tm_v, ld_bar, v_col0 + t.hv * D + h * 64, t.t0, t.b, 0);
    }
  }
  tile_meta<C>(a, t, m);
  ok = mbar_wait(ld_bar, 0, a.err, 101);
  const bool valid = t.p0 + r < t.Ls;
  if (MODE == OUT && !valid) {
    // rows past the clean stream hold other streams' (unwritten) U rows: zero them
#pragma unroll 1
    for (int g = 0; g < 4; ++g) sm_zero32(sm + S::R3, r, g);
  }
  fence_async_smem();
  __syncthreads();

  // ---- KK^T (acc0) and QK^T (acc3) ------------------------------------------------------------------
  if (ok && r == 0) {
    tc_fence_after();
    if (MODE != OUT) mma(acc0, KM(sbase + S::R1), KM(sbase + S::R1), 128, 128, false);
    if (MODE != PREP) mma(acc3, KM(sbase + S::R0), KM(sbase + S::R1), 128, 128, false);
    umma_commit(mma_bar);
  }
  ok = mbar_wait(mma_bar, mph & 1, a.err, 102) && ok;
  ++mph;
  tc_fence_after();
  const int cs = (r / C) * C;
  const int64_t grow0 = (int64_t)t.b * a.T + t.t0;    // global row of tile row 0
  float x[32];

  if (MODE != OUT) {
    // ---- A blocks (fp32, chunk-local columns) and T = (I + A)^-1 ---------------------------------
    {
      float* Af = reinterpret_cast<float*>(sm + S::R4);
      const float Gt = m.G[r], bt = m.beta[r];
      const int sg = m.seg[r];
#pragma unroll 1
      for (int g = WN::g0(); g < WN::g0() + WN::NG; ++g) {
        tm_ld32(acc0, g, x);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int s = 32 * g + i;
          if (s >= cs && s < cs + C)
            Af[af_idx(r, s - cs)] = (s < r && m.seg[s] == sg) ? bt * x[i] * __expf(Gt - m.G[s]) : 0.f;
        }
      }
    }
    __syncthreads();
    invert_column<C>(reinterpret_cast<const float*>(sm + S::R4), sm + S::R3);
    // ---- K~ rows (PREP), Kb = diag(beta carry e^G) K and Vb = diag(beta) V in place ---------------
    {
      const float ks = m.beta[r] * m.carry[r] * __expf(m.G[r]), bs = m.beta[r];
      bf16* kt_row = a.kt + ((grow0 + r) * a.Hv + t.hv) * D;
#pragma unroll 1
      for (int g = 0; g < 4; ++g) {
        sm_ld32(sm + S::R1, r, g, x);
        if (MODE == PREP && valid) gm_st32(kt_row + 32 * g, x, m.kts[r]);
        sm_st32(sm + S::R1, r, g, x, ks);
        sm_ld32(sm + S::R2, r, g, x);
        sm_st32(sm + S::R2, r, g, x, bs);
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    // ---- W = T Kb (acc1); U~ = T Vb (PREP) or U~^T = Vb^T T^T (NOISY) into acc2 ------------------
    if (ok && r == 0) {
      tc_fence_after();
      mma(acc1, KM(sbase + S::R3), MN(sbase + S::R1), 128, 128, false);
      if (MODE == PREP) mma(acc2, KM(sbase + S::R3), MN(sbase + S::R2), 128, 128, false);
      else mma(acc2, MN(sbase + S::R2), KM(sbase + S::R3), 128, 128, false);
      umma_commit(mma_bar);
    }
    ok = mbar_wait(mma_bar, mph & 1, a.err, 103) && ok;
    ++mph;
    tc_fence_after();
    {
      bf16* wn_row = a.wn + ((grow0 + r) * a.Hv + t.hv) * D;
      bf16* ut_row = a.ut + ((grow0 + r) * a.Hv + t.hv) * D;
#pragma unroll 1
      for (int g = 0; g < 4; ++g) {
        tm_ld32(acc1, g, x);
        if (valid) gm_st32(wn_row + 32 * g, x, -1.f);                // -W rows (scan / backward)
        if (MODE == NOISY) sm_st32(sm + S::R4, r, g, x, -1.f);      // -W tile (A blocks are dead)
        if (MODE == PREP) {
          tm_ld32(acc2, g, x);
          if (valid) gm_st32(ut_row + 32 * g, x);
        }
      }
    }
    if (MODE == PREP && r % C == 0 && valid)
      a.gamma[((int64_t)t.b * a.Hv + t.hv) * a.nch + (t.p0 + r) / C] = m.gam[r / C];
  }

  if (MODE != PREP) {
    // ---- Qg = diag(carry e^{Gr}) Q in place (QK^T has completed) ----------------------------------
    {
      const float qs = m.carry[r] * __expf(m.Gr[r]);
#pragma unroll 1
      for (int g = 0; g < 4; ++g) {
        sm_ld32(sm + S::R0, r, g, x);
        sm_st32(sm + S::R0, r, g, x, qs);
      }
    }
    tmem_wait_ld();
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    // ---- per chunk: O^T[:, chunk] = S0^T Qg^T (acc1); NOISY: U^T[:, chunk] += S0^T (-W)^T (acc2) ----
    if (r == 0) {
      const int64_t sb = ((int64_t)t.b * a.Hv + t.hv) * a.nch;
      auto issue = [&](int c) {
        const int buf = c & 1;
        uint8_t* dst = sm + (buf ? S::R5A : S::R1);
        int blk = t.p0 / C + c;
        blk = blk < a.nch ? blk : a.nch - 1;
        const int srow = (int)((sb + blk) * D);
        mbar_expect_tx(&st_bar[buf], TILE);
        tma_load_4d(dst, &tm_st, &st_bar[buf], 0, srow, 0, 0);
        tma_load_4d(dst + SUB, &tm_st, &st_bar[buf], 64, srow, 0, 0);
      };
      // buffer 0 aliases K / Kb, whose MMAs completed above
      issue(0);
      if (NCK > 1) issue(1);
      uint32_t sph[2] = {0, 0};
      uint32_t lph = mph;
      for (int c = 0; c < NCK; ++c) {
        const int buf = c & 1;
        if (ok) ok = mbar_wait(&st_bar[buf], sph[buf] & 1, a.err, 104);
        ++sph[buf];
        if (ok) {
          tc_fence_after();
          const uint32_t sbuf = sbase + (buf ? S::R5A : S::R1);
          mma(acc1 + c * C, MN(sbuf), KM(sbase + S::R0, c * C), C, 128, false);
          if (MODE == NOISY) mma(acc2 + c * C, MN(sbuf), KM(sbase + S::R4, c * C), C, 128, true);
        }
        umma_commit(mma_bar);
        if (ok) ok = mbar_wait(mma_bar, lph & 1, a.err, 105);
        ++lph;
        if (c + 2 < NCK) {
          if (ok) issue(c + 2);
          else ++sph[buf];
        }
      }
    }
    __syncthreads();
    mph += NCK;
    tc_fence_after();
    // ---- P (window of acc3) into R2; NOISY: U^T (acc2; row r = value column r) into R3 + U rows -----
    {
      const float Gr = m.Gr[r];
      const int rd = m.rd[r], sg = m.seg[r];
#pragma unroll 1
      for (int g = 0; g < 4; ++g) {
        if (g < WN::g0() || g >= WN::g0() + WN::NG) {
          sm_zero32(sm + S::R2, r, g);
          continue;
        }
        tm_ld32(acc3, g, x);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int s = 32 * g + i;
          const bool on = (s >= cs) && (s <= rd) && (m.seg[s] == sg);
          x[i] = on ? x[i] * __expf(Gr - m.G[s]) : 0.f;
        }
        sm_st32(sm + S::R2, r, g, x);
      }
    }
    if (MODE == NOISY) {
      bf16* ub = a.u + grow0 * a.Hv * D + t.hv * D + r;
      const int nv = min(TR, t.Ls - t.p0);
#pragma unroll 1
      for (int g = 0; g < 4; ++g) {
        tm_ld32(acc2, g, x);
        sm_st32(sm + S::R3, r, g, x);
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (32 * g + i < nv) ub[(int64_t)(32 * g + i) * a.Hv * D] = __float2bfloat16(x[i]);
      }
    }
    tmem_wait_ld();
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    // ---- O^T += U^T P^T -----------------------------------------------------------------------------
    if (ok && r == 0) {
      tc_fence_after();
      if (MODE == NOISY) mma(acc1, KM(sbase + S::R3), KM(sbase + S::R2), 128, 128, true);
      else mma(acc1, MN(sbase + S::R3), KM(sbase + S::R2), 128, 128, true);
      umma_commit(mma_bar);
    }
    ok = mbar_wait(mma_bar, mph & 1, a.err, 106) && ok;
    ++mph;
    tc_fence_after();
    // ---- O: row r of acc1 is value column r; stage transposed in R0, then rows to global ------------
#pragma unroll 1
    for (int g = 0; g < 4; ++g) {
      tm_ld32(acc1, g, x);
      sm_st_col32(sm + S::R0, r, g, x);
    }
    __syncthreads();
    if (valid) {
      bf16* orow = a.o + (grow0 + r) * (int64_t)(a.Hv * D) + t.hv * D;
#pragma unroll 1
      for (int g = 0; g < 4; ++g) {
        sm_ld32(sm + S::R0, r, g, x);
        gm_st32(orow + 32 * g, x);
      }
    }
  }
  tmem_wait_ld();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (r < 32) tmem_dealloc(tmem, 512);
}

// ---- scan: clean chunks in order, per (row, value head) ---------------------------------------------
// Shared memory: the state as a bf16 tile (S[k][v]), a double-buffered stage of C-row tiles
// (-W, K~, U~ by TMA: two [C][64] halves each), and U as the B operand [v][t] (one [128][64] half,
// first C columns used).  TMEM: the fp32 state (128 columns) and U^T (C columns).
template <int C>
struct ScanSmem {
  static constexpr int SB = 0;
  static constexpr int STAGE_TILE = C * 256;
  static constexpr int STG = SB + TILE;
  static constexpr int STG_BYTES = 3 * STAGE_TILE;
  static constexpr int UB = STG + 2 * STG_BYTES;
  static constexpr int BARS = UB + SUB;
  static constexpr int TOTAL = BARS + 64;
};

template <int C>
__global__ void __launch_bounds__(NT, 1) scan_kernel(const __grid_constant__ CUtensorMap tm_wn,
                                                     const __grid_constant__ CUtensorMap tm_kt,
                                                     const __grid_constant__ CUtensorMap tm_ut, const Args a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  using S = ScanSmem<C>;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + S::BARS);
  uint64_t* ld_bar = bars;       // two stage buffers
  uint64_t* mma_bar = bars + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 4);
  const int hv = blockIdx.x, b = blockIdx.y, r = threadIdx.x;
  const int Lc = clean_len(a);
  const int nch = a.nch;
  if (r == 0) {
    mbar_init(&ld_bar[0], 1);
    mbar_init(&ld_bar[1], 1);
    mbar_init(mma_bar, 1);
    fence_barrier_init();
  }
  if (r < 32) tmem_alloc(tmem_slot, 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t accS = tmem, accU = tmem + 128;
  const uint32_t sbase = smem_addr(sm);
  auto stage = [&](int buf, int which) -> uint8_t* { return sm + S::STG + buf * S::STG_BYTES + which * S::STAGE_TILE; };
  auto issue = [&](int c) {
    const int buf = c & 1;
    mbar_expect_tx(&ld_bar[buf], 3 * S::STAGE_TILE);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      tma_load_4d(stage(buf, 0) + h * C * 128, &tm_wn, &ld_bar[buf], h * 64, hv, c * C, b);
      tma_load_4d(stage(buf, 1) + h * C * 128, &tm_kt, &ld_bar[buf], h * 64, hv, c * C, b);
      tma_load_4d(stage(buf, 2) + h * C * 128, &tm_ut, &ld_bar[buf], h * 64, hv, c * C, b);
    }
  };
  if (r == 0) {
    prefetch_tmap(&tm_wn);
    prefetch_tmap(&tm_kt);
    prefetch_tmap(&tm_ut);
    issue(0);
    if (nch > 1) issue(1);
  }
  float x[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) x[i] = 0.f;
#pragma unroll 1
  for (int g = 0; g < 4; ++g) tm_st32(accS, g, x);
  tmem_wait_st();
  bool ok = true;
  uint32_t lph[2] = {0, 0}, mph = 0;
  const int64_t srow0 = ((int64_t)b * a.Hv + hv) * nch;
  for (int c = 0; c < nch && ok; ++c) {
    const int buf = c & 1;
    // the state entering chunk c: bf16 copy into SB and the checkpoint, then scaled by the chunk decay
    tc_fence_after();
    {
      const float gam = a.gamma[srow0 + c];
      bf16* ck = a.ckpt + ((srow0 + c) * D + r) * D;
#pragma unroll 1
      for (int g = 0; g < 4; ++g) {
        tm_ld32(accS, g, x);
        sm_st32(sm + S::SB, r, g, x);
        gm_st32(ck + 32 * g, x);
#pragma unroll
        for (int i = 0; i < 32; ++i) x[i] *= gam;
        tm_st32(accS, g, x);
      }
      tmem_wait_st();
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    ok = mbar_wait(&ld_bar[buf], lph[buf] & 1, a.err, 111);
    ++lph[buf];
    ok = __syncthreads_and(ok) != 0;    // every thread leaves the loop at the same chunk
    if (!ok) break;
    // MMA1: U^T[v][t] = S^T (-W)^T  (A = S: MN-major; B = -W stage tile: K-major, N = C rows)
    if (r == 0) {
      tc_fence_after();
      mma(accU, MN(sbase + S::SB), KM(smem_addr(stage(buf, 0)), 0, 0, C * 128), C, 128, false);
      umma_commit(mma_bar);
    }
    ok = mbar_wait(mma_bar, mph & 1, a.err, 112);
    ++mph;
    tc_fence_after();
    // U[t][v] = U~[t][v] + acc (thread r = value column v); zero past the stream end
    float u[C];
#pragma unroll
    for (int j = 0; j < C / 16; ++j) {
      uint32_t v[16];
      tmem_ld16(accU + lane_base() + 16 * j, v);
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 16; ++i) u[16 * j + i] = __uint_as_float(v[i]);
    }
    {
      const uint8_t* ut = stage(buf, 2) + (r >> 6) * C * 128;
      const int64_t row0 = (int64_t)b * a.T + (int64_t)c * C;
#pragma unroll
      for (int tt = 0; tt < C; ++tt) {
        const float uv = __bfloat162float(*reinterpret_cast<const bf16*>(ut + sw128_offset(tt, r & 63))) + u[tt];
        const bool in = c * C + tt < Lc;
        u[tt] = in ? uv : 0.f;
        if (in) a.u[((row0 + tt) * a.Hv + hv) * D + r] = __float2bfloat16(uv);
      }
      uint8_t* ub = sm + S::UB;
#pragma unroll
      for (int j = 0; j < C / 8; ++j) {
        uint4 v;
        v.x = pack_bf2(u[8 * j], u[8 * j + 1]); v.y = pack_bf2(u[8 * j + 2], u[8 * j + 3]);
        v.z = pack_bf2(u[8 * j + 4], u[8 * j + 5]); v.w = pack_bf2(u[8 * j + 6], u[8 * j + 7]);
        *reinterpret_cast<uint4*>(ub + sw128_offset(r, 8 * j)) = v;
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    // MMA2: S[k][v] += K~^T U  (A = K~ stage tile: MN-major over its C rows; B = Ub: K-major)
    if (r == 0) {
      tc_fence_after();
      mma(accS, MN(smem_addr(stage(buf, 1)), 0, C * 128), KM(sbase + S::UB), 128, C, true);
      umma_commit(mma_bar);
    }
    ok = mbar_wait(mma_bar, mph & 1, a.err, 113) && ok;
    ++mph;
    ok = __syncthreads_and(ok) != 0;
    // the stage buffer is free: prefetch chunk c + 2
    if (ok && r == 0 && c + 2 < nch) issue(c + 2);
  }
  tc_fence_after();
  if (ok && a.final_state != nullptr) {
    float* f = a.final_state + (((int64_t)b * a.Hv + hv) * D + r) * D;
#pragma unroll 1
    for (int g = 0; g < 4; ++g) {
      tm_ld32(accS, g, x);
#pragma unroll
      for (int i = 0; i < 32; i += 4)
        *reinterpret_cast<float4*>(f + 32 * g + i) = make_float4(x[i], x[i + 1], x[i + 2], x[i + 3]);
    }
  }
  tmem_wait_ld();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (r < 32) tmem_dealloc(tmem, 256);
}

// ---- prep: bf16 L2-normalised q (times scale) / k, log-decay and beta -------------------------------
__global__ void chunk_prep_kernel(const bf16* mixed, int64_t ldm, const bf16* ga, const bf16* gbeta, int64_t ldg,
                                  const float* A_log, const float* dt_bias, int rows, int Hk, int Hv, float scale,
                                  bf16* qk, float* gb) {
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int per_row = 2 * Hk + 1;
  if (gw >= (int64_t)rows * per_row) return;
  const int64_t row = gw / per_row;
  const int w = (int)(gw % per_row);
  if (w < 2 * Hk) {
    const int hk = w >> 1, isk = w & 1;
    const bf16* src = mixed + row * ldm + isk * Hk * D + hk * D + lane * 4;
    const uint2 raw = *reinterpret_cast<const uint2*>(src);
    const bf16* e = reinterpret_cast<const bf16*>(&raw);
    float v[4], ss = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[i] = __bfloat162float(e[i]);
      ss += v[i] * v[i];
    }
    ss = warp_sum(ss);
    const float rn = rsqrtf(ss + 1e-6f) * (isk ? 1.f : scale);
    uint2 o;
    o.x = pack_bf2(v[0] * rn, v[1] * rn);
    o.y = pack_bf2(v[2] * rn, v[3] * rn);
    *reinterpret_cast<uint2*>(qk + ((row * Hk + hk) * 2 + isk) * D + lane * 4) = o;
  } else {
    for (int h = lane; h < Hv; h += 32) {
      const float av = __bfloat162float(ga[row * ldg + h]) + dt_bias[h];
      const float bv = __bfloat162float(gbeta[row * ldg + h]);
      const float sp = av > 20.f ? av : log1pf(expf(av));
      gb[(row * Hv + h) * 2] = -expf(A_log[h]) * sp;
      gb[(row * Hv + h) * 2 + 1] = 1.f / (1.f + expf(-bv));
    }
  }
}

template <int C>
static int launch_fwd(const GdnChunkParams& p, const Args& a, cudaStream_t st) {
  CUtensorMap m_qk, m_v, m_u, m_st, m_wn, m_kt, m_ut;
  if (!map_heads(&m_qk, p.qk, p.B, p.T, 2 * p.Hk, TR)) return -2;
  if (!map_cols(&m_v, p.mixed, p.B, p.T, 2 * p.Hk * D + p.Hv * D, p.ldm, TR)) return -3;
  if (!map_heads(&m_u, p.u, p.B, p.T, p.Hv, TR)) return -4;
  if (!map_cols(&m_st, p.ckpt, 1, p.B * p.Hv * p.nch * D, D, D, 128)) return -5;
  if (!map_heads(&m_wn, p.wn, p.B, p.T, p.Hv, C)) return -6;
  if (!map_heads(&m_kt, p.kt, p.B, p.T, p.Hv, C)) return -7;
  if (!map_heads(&m_ut, p.ut, p.B, p.T, p.Hv, C)) return -8;
  const int v_col0 = 2 * p.Hk * D;
  const int lsmem = LocalSmem::TOTAL + 1024, ssmem = ScanSmem<C>::TOTAL + 1024;
  static bool init = false;
  if (!init) {
    cudaFuncSetAttribute(local_kernel<PREP, C>, cudaFuncAttributeMaxDynamicSharedMemorySize, lsmem);
    cudaFuncSetAttribute(local_kernel<NOISY, C>, cudaFuncAttributeMaxDynamicSharedMemorySize, lsmem);
    cudaFuncSetAttribute(local_kernel<OUT, C>, cudaFuncAttributeMaxDynamicSharedMemorySize, lsmem);
    cudaFuncSetAttribute(scan_kernel<C>, cudaFuncAttributeMaxDynamicSharedMemorySize, ssmem);
    init = true;
  }
  const int Lc = p.mode ? p.L : p.T;
  const int tiles = (Lc + TR - 1) / TR;
  local_kernel<PREP, C><<<dim3(tiles, p.Hv, p.B), NT, lsmem, st>>>(m_qk, m_v, m_u, m_st, a, v_col0);
  scan_kernel<C><<<dim3(p.Hv, p.B), NT, ssmem, st>>>(m_wn, m_kt, m_ut, a);
  local_kernel<OUT, C><<<dim3(tiles, p.Hv, p.B), NT, lsmem, st>>>(m_qk, m_v, m_u, m_st, a, v_col0);
  if (p.mode) local_kernel<NOISY, C><<<dim3(tiles, p.Hv, p.B * p.V), NT, lsmem, st>>>(m_qk, m_v, m_u, m_st, a, v_col0);
  return 0;
}

}  // namespace gdnc

using namespace gdnc;

int gdn_chunk_fwd(const GdnChunkParams& p, cudaStream_t st) {
  const int rows = p.B * p.T;
  {
    const int64_t warps = (int64_t)rows * (2 * p.Hk + 1);
    chunk_prep_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, st>>>(
        p.mixed, p.ldm, p.ga, p.gbeta, p.ldg, p.A_log, p.dt_bias, rows, p.Hk, p.Hv, p.scale, p.qk, p.gb);
  }
  Args a{};
  a.B = p.B; a.T = p.T; a.Hk = p.Hk; a.Hv = p.Hv; a.mode = p.mode; a.L = p.L; a.V = p.V;
  a.nch = p.nch; a.tok_clean = p.causal_clean; a.tok_noisy = p.causal_noisy; a.doc = p.doc; a.gb = p.gb;
  a.o = p.o; a.ckpt = p.ckpt; a.gamma = p.gamma; a.final_state = p.final_state;
  a.wn = p.wn; a.ut = p.ut; a.kt = p.kt; a.u = p.u; a.err = p.err;
  int rc;
  switch (p.C) {
    case 16: rc = launch_fwd<16>(p, a, st); break;
    case 32: rc = launch_fwd<32>(p, a, st); break;
    case 64: rc = launch_fwd<64>(p, a, st); break;
    default: return -1;
  }
  if (rc != 0) return rc;
  return cudaGetLastError() == cudaSuccess ? 0 : -9;
}

}  // namespace trida
