// Backward of the chunked gated-delta rule on tcgen05 (sm_100a).  The formulas are the explicit
// chunk backward stated in trida_stack_b200/ops/gdn_chunked.py (chunk_bwd), on the same 128-row
// tiles and tile algebra as the forward (gdn_chunk.cuh).  Per chunk, with dS1 the gradient of the
// state after the chunk (zero for noisy blocks and for the last clean chunk):
//     dU  = P^T dO + K~ dS1                      dP = dO U^T (masked),  dPE = dP e^{Gr_t - G_s}
//     dQ  = dPE K + diag(carry e^Gr) dO S0^T     dW = -dU S0^T
//     dT  = dU Vb^T + dW Kb^T,  dA = -T^T dT T^T (strict lower, same segment)
//     dV  = diag(beta) T^T dU,  dKb = T^T dW
//     dK  = dPE^T Q + dAE K + dAE^T K + diag(beta carry e^G) dKb + diag(kts) dS1 U^T-rows
//     dS0 = (carry e^Gr Q)^T dO - W^T dU + gamma dS1
// and the log-decay / beta gradients from row dots (the column sums of dP.P and dA.A are
// k_s . (column-part of dK_s), so they come out of lanes-s products without a transpose).
//
// Launch order per layer (one stream):
//   bwd0  (every tile)      : P, dU0 = P^T dO (noisy rows: dU itself), carry e^Gr q rows (clean).
//   ds0   (two-stream)      : per clean block and value head, the noisy views' gradient w.r.t. the
//                             clean state at the block start (Q^T dOg - W^T dU summed over views).
//   scanb (clean stream)    : reverse over chunks: dS (fp32 in TMEM), dU of the clean rows, and
//                             the bf16 dS1 of every chunk.
//   bwd1  (every tile)      : T, dPE, dQ, dW, dT, dA (rows of dPE, dAE, dW, T for bwd2).
//   bwd2  (every tile)      : dV, dKb, dK (+ the end-state term of clean chunks), d beta, dg.
//   post  (every row)       : sum over the value heads of a key head, q/k L2-norm and gate backward.
#include "gdn_chunk.cuh"

namespace trida {
namespace gdnc {

using namespace trida::sm100;

constexpr int RED = 2 * D + 4;   // per (row, value head): dq | dk | dbeta | dg | pad

// Stream geometry of the tile of blockIdx (stream index from blockIdx.z = b * nstreams + s).
__device__ __forceinline__ TileGeo tile_geo(const Args& a) {
  TileGeo t;
  const int ns = a.mode ? 1 + a.V : 1;
  t.hv = blockIdx.y;
  t.hk = t.hv / (a.Hv / a.Hk);
  t.b = blockIdx.z / ns;
  t.stream = blockIdx.z % ns;
  t.Ls = clean_len(a);
  t.p0 = blockIdx.x * TR;
  t.t0 = t.stream * a.L + t.p0;
  t.tok = (t.stream == 0) ? (a.mode == 0 || a.tok_clean) : a.tok_noisy;
  return t;
}

__device__ __forceinline__ int64_t grow(const Args& a, const TileGeo& t, int r) {
  return (int64_t)t.b * a.T + t.t0 + r;
}

// thread 0: a 128-row tile of per-head rows (two halves)
__device__ __forceinline__ void load_rows(uint8_t* dst, const CUtensorMap* m, uint64_t* bar, int h, int t0, int b) {
  tma_load_4d(dst, m, bar, 0, h, t0, b);
  tma_load_4d(dst + SUB, m, bar, 64, h, t0, b);
}
__device__ __forceinline__ void load_cols(uint8_t* dst, const CUtensorMap* m, uint64_t* bar, int col, int t0, int b) {
  tma_load_4d(dst, m, bar, col, t0, b, 0);
  tma_load_4d(dst + SUB, m, bar, col + 64, t0, b, 0);
}
__device__ __forceinline__ void load_state(uint8_t* dst, const CUtensorMap* m, uint64_t* bar, int row) {
  tma_load_4d(dst, m, bar, 0, row, 0, 0);
  tma_load_4d(dst + SUB, m, bar, 64, row, 0, 0);
}

#define SYNC_FOR_MMA()   \
  do {                   \
    tmem_wait_ld();      \
    fence_async_smem();  \
    tc_fence_before();   \
    __syncthreads();     \
  } while (0)

#define WAIT_MMA(code)                                        \
  do {                                                        \
    ok = mbar_wait(mma_bar, mph & 1, a.err, (code)) && ok;    \
    ++mph;                                                    \
    tc_fence_after();                                         \
  } while (0)

#define WAIT_LD(code)                                         \
  do {                                                        \
    ok = mbar_wait(ld_bar, lph & 1, a.err, (code)) && ok;     \
    ++lph;                                                    \
  } while (0)

struct BwdSmem {
  static constexpr int S0 = 0, S1 = TILE, S2 = 2 * TILE, S3 = 3 * TILE, S4 = 4 * TILE, S5 = 5 * TILE;
  static constexpr int META = 6 * TILE;
  static constexpr int RED = META + Meta::BYTES;        // colsum scratch [4][128] + dG [128] + misc
  static constexpr int BARS = RED + (4 * 128 + 3 * 128 + 8) * 4;
  static constexpr int TOTAL = BARS + 64;
};

struct BwdMaps {
  CUtensorMap qk, d_o, u, du, st, dst, v;   // v: conv output columns
};

// ---- bwd0: P, dU0 = P^T dO, qg rows ------------------------------------------------------------------
template <int C>
__global__ void __launch_bounds__(NT, 1) bwd0_kernel(const __grid_constant__ CUtensorMap tm_qk,
                                                     const __grid_constant__ CUtensorMap tm_do, const Args a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  using S = BwdSmem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + S::BARS);
  uint64_t* ld_bar = bars;
  uint64_t* mma_bar = bars + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2);
  const Meta m = carve_meta(sm + S::META);
  const int r = threadIdx.x;
  const TileGeo t = tile_geo(a);
  if (r == 0) {
    mbar_init(ld_bar, 1);
    mbar_init(mma_bar, 1);
    fence_barrier_init();
  }
  if (r < 32) tmem_alloc(tmem_slot, 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t accP = tmem, accU = tmem + 128;
  const uint32_t sbase = smem_addr(sm);
  uint32_t mph = 0, lph = 0;
  bool ok = true;
  if (r == 0) {
    mbar_expect_tx(ld_bar, 3 * TILE);
    load_rows(sm + S::S0, &tm_qk, ld_bar, 2 * t.hk, t.t0, t.b);
    load_rows(sm + S::S1, &tm_qk, ld_bar, 2 * t.hk + 1, t.t0, t.b);
    load_cols(sm + S::S2, &tm_do, ld_bar, t.hv * D, t.t0, t.b);
  }
  tile_meta<C>(a, t, m);
  WAIT_LD(201);
  if (ok && r == 0) {
    tc_fence_after();
    mma(accP, KM(sbase + S::S0), KM(sbase + S::S1), 128, 128, false);
    umma_commit(mma_bar);
  }
  WAIT_MMA(202);
  const int cs = (r / C) * C;
  const bool valid = t.p0 + r < t.Ls;
  using WN = Win<C>;
  float x[32];
  {
    const float Gr = m.Gr[r];
    const int rd = m.rd[r], sg = m.seg[r];
#pragma unroll 1
    for (int g = 0; g < 4; ++g) {
      if (g < WN::g0() || g >= WN::g0() + WN::NG) {
        sm_zero32(sm + S::S3, r, g);
        continue;
      }
      tm_ld32(accP, g, x);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int s = 32 * g + i;
        const bool on = (s >= cs) && (s <= rd) && (m.seg[s] == sg) && valid;
        x[i] = on ? x[i] * __expf(Gr - m.G[s]) : 0.f;
      }
      sm_st32(sm + S::S3, r, g, x);
    }
  }
  // zero dO rows past the stream (other streams' rows must not leak into dU)
  if (!valid) {
#pragma unroll 1
    for (int g = 0; g < 4; ++g) sm_zero32(sm + S::S2, r, g);
  }
  SYNC_FOR_MMA();
  // dU0^T[v][s] = sum_t dO[t][v] P[t][s]
  if (ok && r == 0) {
    tc_fence_after();
    mma(accU, MN(sbase + S::S2), MN(sbase + S::S3), 128, 128, false);
    umma_commit(mma_bar);
  }
  // clean stream: the carry e^{Gr} q rows for the scan
  if (t.stream == 0 && valid) {
    bf16* dst = a.qg + (grow(a, t, r) * a.Hv + t.hv) * D;
    const float qs = m.carry[r] * __expf(m.Gr[r]);
#pragma unroll 1
    for (int g = 0; g < 4; ++g) {
      sm_ld32(sm + S::S0, r, g, x);
      gm_st32(dst + 32 * g, x, qs);
    }
  }
  WAIT_MMA(203);
  {
    bf16* dst = (t.stream == 0 ? a.du0 : a.du) + grow(a, t, 0) * a.Hv * D + t.hv * D + r;
    const int nv = min(TR, t.Ls - t.p0);
#pragma unroll 1
    for (int g = 0; g < 4; ++g) {
      tm_ld32(accU, g, x);   // row r = value column r over the tile rows 32g..
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (32 * g + i < nv) dst[(int64_t)(32 * g + i) * a.Hv * D] = __float2bfloat16(x[i]);
    }
  }
  tmem_wait_ld();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (r < 32) tmem_dealloc(tmem, 256);
}

// ---- ds0: noisy gradient w.r.t. the clean state at each block start --------------------------------
// Grid (nch, Hv, B).  Stage tiles of C rows per view: Q (key head), dO, -W, dU.
template <int C>
__global__ void __launch_bounds__(NT, 1) ds0_kernel(const __grid_constant__ CUtensorMap tm_qk,
                                                    const __grid_constant__ CUtensorMap tm_do,
                                                    const __grid_constant__ CUtensorMap tm_wn,
                                                    const __grid_constant__ CUtensorMap tm_du, const Args a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int ST = C * 256;                  // one C-row stage tile
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + 4 * ST);
  uint64_t* ld_bar = bars;
  uint64_t* mma_bar = bars + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2);
  float* sc = reinterpret_cast<float*>(bars + 4);   // [C] dO row scales
  const int c = blockIdx.x, hv = blockIdx.y, b = blockIdx.z, r = threadIdx.x;
  const int hk = hv / (a.Hv / a.Hk);
  if (r == 0) {
    mbar_init(ld_bar, 1);
    mbar_init(mma_bar, 1);
    fence_barrier_init();
  }
  if (r < 32) tmem_alloc(tmem_slot, 128);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t acc = *tmem_slot;
  const uint32_t sbase = smem_addr(sm);
  uint32_t mph = 0, lph = 0;
  bool ok = true;
  const bool carry = a.doc == nullptr || a.doc[(int64_t)b * a.L + c * C] == 0;
  for (int v = 0; v < a.V; ++v) {
    const int t0 = (1 + v) * a.L + c * C;
    if (r == 0) {
      mbar_expect_tx(ld_bar, 4 * ST);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        tma_load_4d(sm + 0 * ST + h * C * 128, &tm_qk, ld_bar, h * 64, 2 * hk, t0, b);
        tma_load_4d(sm + 1 * ST + h * C * 128, &tm_do, ld_bar, hv * D + h * 64, t0, b, 0);
        tma_load_4d(sm + 2 * ST + h * C * 128, &tm_wn, ld_bar, h * 64, hv, t0, b);
        tma_load_4d(sm + 3 * ST + h * C * 128, &tm_du, ld_bar, h * 64, hv, t0, b);
      }
    }
    // dO row scales carry e^{Gr}: one segment per noisy block
    if (r == 0) {
      float G = 0.f;
      for (int j = 0; j < C; ++j) {
        G += a.gb[(((int64_t)b * a.T + t0 + j) * a.Hv + hv) * 2];
        sc[j] = G;
      }
      const float Gl = sc[C - 1];
      for (int j = 0; j < C; ++j) sc[j] = carry ? __expf(a.tok_noisy ? sc[j] : Gl) : 0.f;
    }
    WAIT_LD(211);
    __syncthreads();
    if (r < C) {
      uint8_t* row = sm + 1 * ST;
      const float s = sc[r];
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          uint4* p = reinterpret_cast<uint4*>(row + h * C * 128 + sw128_offset(r, 8 * j));
          uint4 q = *p;
          uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            float2 f = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&w[i]));
            w[i] = pack_bf2(f.x * s, f.y * s);
          }
          *p = make_uint4(w[0], w[1], w[2], w[3]);
        }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    if (ok && r == 0) {
      tc_fence_after();
      // acc[k][v] += sum_t Q[t][k] dOg[t][v] + sum_t (-W)[t][k] dU[t][v]
      mma(acc, MN(sbase + 0 * ST, 0, C * 128), MN(sbase + 1 * ST, 0, C * 128), 128, C, v > 0);
      mma(acc, MN(sbase + 2 * ST, 0, C * 128), MN(sbase + 3 * ST, 0, C * 128), 128, C, true);
      umma_commit(mma_bar);
    }
    WAIT_MMA(212);
    ok = __syncthreads_and(ok) != 0;
    if (!ok) break;
  }
  {
    float x[32];
    bf16* dst = a.ds0 + ((((int64_t)b * a.Hv + hv) * a.nch + c) * D + r) * D;
#pragma unroll 1
    for (int g = 0; g < 4; ++g) {
      tm_ld32(acc, g, x);
      gm_st32(dst + 32 * g, x, ok ? 1.f : 0.f);
    }
  }
  tmem_wait_ld();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (r < 32) tmem_dealloc(acc, 128);
}

// ---- scanb: reverse over the clean chunks --------------------------------------------------------
// Stage per chunk (C rows each): K~, qg, dO, -W, dU0 (+ the noisy state-gradient tile for the
// two-stream layout).  TMEM: dS (128 columns), dU^T (C columns).
template <int C, bool NOISY>
struct ScanbSmem {
  static constexpr int ST = C * 256;
  static constexpr int STAGE = 5 * ST + (NOISY ? TILE : 0);
  static constexpr int NST = (C == 64 && NOISY) ? 1 : 2;
  static constexpr int SB = 0;                     // dS as bf16 [k][v]
  static constexpr int STG = TILE;
  static constexpr int UB = STG + NST * STAGE;     // dU as B operand [v][t]
  static constexpr int BARS = UB + SUB;
  static constexpr int TOTAL = BARS + 64;
};

template <int C, bool NOISY>
__global__ void __launch_bounds__(NT, 1) scanb_kernel(const __grid_constant__ CUtensorMap tm_kt,
                                                      const __grid_constant__ CUtensorMap tm_qg,
                                                      const __grid_constant__ CUtensorMap tm_do,
                                                      const __grid_constant__ CUtensorMap tm_wn,
                                                      const __grid_constant__ CUtensorMap tm_du0,
                                                      const __grid_constant__ CUtensorMap tm_ds0, const Args a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  using S = ScanbSmem<C, NOISY>;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + S::BARS);
  uint64_t* ld_bar = bars;        // [2]
  uint64_t* mma_bar = bars + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 4);
  const int hv = blockIdx.x, b = blockIdx.y, r = threadIdx.x;
  const int Lc = clean_len(a), nch = a.nch;
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
  const uint32_t lane_off = (uint32_t)(32 * (r >> 5)) << 16;
  const uint32_t sbase = smem_addr(sm);
  const int64_t srow0 = ((int64_t)b * a.Hv + hv) * nch;
  auto stage = [&](int c, int which) -> uint8_t* {
    return sm + S::STG + (S::NST == 1 ? 0 : (c & 1)) * S::STAGE + which * S::ST;
  };
  auto issue = [&](int c) {
    uint64_t* bar = &ld_bar[S::NST == 1 ? 0 : (c & 1)];
    mbar_expect_tx(bar, S::STAGE);
    const int t0 = c * C;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      tma_load_4d(stage(c, 0) + h * C * 128, &tm_kt, bar, h * 64, hv, t0, b);
      tma_load_4d(stage(c, 1) + h * C * 128, &tm_qg, bar, h * 64, hv, t0, b);
      tma_load_4d(stage(c, 2) + h * C * 128, &tm_do, bar, hv * D + h * 64, t0, b, 0);
      tma_load_4d(stage(c, 3) + h * C * 128, &tm_wn, bar, h * 64, hv, t0, b);
      tma_load_4d(stage(c, 4) + h * C * 128, &tm_du0, bar, h * 64, hv, t0, b);
    }
    if (NOISY) {
      tma_load_4d(stage(c, 5), &tm_ds0, bar, 0, (int)((srow0 + c) * D), 0, 0);
      tma_load_4d(stage(c, 5) + SUB, &tm_ds0, bar, 64, (int)((srow0 + c) * D), 0, 0);
    }
  };
  if (r == 0) {
    issue(nch - 1);
    if (S::NST == 2 && nch > 1) issue(nch - 2);
  }
  float x[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) x[i] = 0.f;
#pragma unroll 1
  for (int g = 0; g < 4; ++g) tm_st32(accS, g, x);
  tmem_wait_st();
  bool ok = true;
  uint32_t lph[2] = {0, 0}, mph = 0;
  for (int c = nch - 1; c >= 0 && ok; --c) {
    const int buf = S::NST == 1 ? 0 : (c & 1);
    ok = mbar_wait(&ld_bar[buf], lph[buf] & 1, a.err, 221);
    ++lph[buf];
    ok = __syncthreads_and(ok) != 0;
    if (!ok) break;
    // dS1 of chunk c: bf16 into SB and the checkpoint; then dS <- gamma dS + noisy(c)
    tc_fence_after();
    {
      const float gam = a.gamma[srow0 + c];
      bf16* ck = a.dckpt + ((srow0 + c) * D + r) * D;
      float y[32];
#pragma unroll 1
      for (int g = 0; g < 4; ++g) {
        tm_ld32(accS, g, x);
        sm_st32(sm + S::SB, r, g, x);
        gm_st32(ck + 32 * g, x);
        if (NOISY) sm_ld32(stage(c, 5), r, g, y);
#pragma unroll
        for (int i = 0; i < 32; ++i) x[i] = x[i] * gam + (NOISY ? y[i] : 0.f);
        tm_st32(accS, g, x);
      }
      tmem_wait_st();
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    if (r == 0) {
      tc_fence_after();
      // dU^T[v][t] = sum_k dS1[k][v] K~[t][k]
      mma(accU, MN(sbase + S::SB), KM(smem_addr(stage(c, 0)), 0, 0, C * 128), C, 128, false);
      // dS += Qg^T dO
      mma(accS, MN(smem_addr(stage(c, 1)), 0, C * 128), MN(smem_addr(stage(c, 2)), 0, C * 128), 128, C, true);
      umma_commit(mma_bar);
    }
    ok = mbar_wait(mma_bar, mph & 1, a.err, 222) && ok;
    ++mph;
    tc_fence_after();
    float u[C];
#pragma unroll
    for (int j = 0; j < C / 16; ++j) {
      uint32_t v[16];
      tmem_ld16(accU + lane_off + 16 * j, v);
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 16; ++i) u[16 * j + i] = __uint_as_float(v[i]);
    }
    {
      const uint8_t* du0 = stage(c, 4) + (r >> 6) * C * 128;
      const int64_t row0 = (int64_t)b * a.T + (int64_t)c * C;
#pragma unroll
      for (int tt = 0; tt < C; ++tt) {
        const float uv = __bfloat162float(*reinterpret_cast<const bf16*>(du0 + sw128_offset(tt, r & 63))) + u[tt];
        const bool in = c * C + tt < Lc;
        u[tt] = in ? uv : 0.f;
        if (in) a.du[((row0 + tt) * a.Hv + hv) * D + r] = __float2bfloat16(uv);
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
    if (r == 0) {
      tc_fence_after();
      // dS += (-W)^T dU
      mma(accS, MN(smem_addr(stage(c, 3)), 0, C * 128), KM(sbase + S::UB), 128, C, true);
      umma_commit(mma_bar);
    }
    ok = mbar_wait(mma_bar, mph & 1, a.err, 223) && ok;
    ++mph;
    ok = __syncthreads_and(ok) != 0;
    if (ok && r == 0) {
      const int nxt = (S::NST == 1) ? c - 1 : c - 2;
      if (nxt >= 0) issue(nxt);
    }
  }
  tmem_wait_ld();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (r < 32) tmem_dealloc(tmem, 256);
}

// Decay gradient of pair terms.  A factor Z_ts proportional to exp(G_lim(t) - G_s) contains g_j
// for s < j <= lim(t), so the decay gradient of position j is sum_{t : lim(t) >= j} sum_{s < j}
// dZ_ts Z_ts: each pair enters once and nothing cancels (the equivalent row-sum-minus-column-sum
// form subtracts two large, differently rounded terms).  Pair terms are block diagonal, so a row's
// pairs lie in its window; thread t walks its window groups with a running prefix over s and the
// masked prefixes are summed over the rows of the window: inside the warp by warp_colsum32, across
// the window's warps (C = 64) through red[warp][column].
template <int C>
struct PairSum {
  float run = 0.f;
  // x: dZ . Z for columns 32g.. of this row; lim: the row's last position whose decay it carries
  __device__ void group(float (&x)[32], int g, int lim, float* red) {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const float v = x[i];
      x[i] = (lim >= 32 * g + i) ? run : 0.f;
      run += v;
    }
    const float cs = warp_colsum32(x);
    red[(threadIdx.x >> 5) * 128 + 32 * g + (threadIdx.x & 31)] = cs;
  }
  // after a CTA barrier: thread j's total over the warps of its window
  __device__ static float total(const float* red) {
    using WN = Win<C>;
    const int j = threadIdx.x, w0 = (j / WN::W) * (WN::W / 32);
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < WN::W / 32; ++w) s += red[(w0 + w) * 128 + j];
    return s;
  }
};

// ---- bwd1: T, dPE, dQ, dW, dT, dA and the pair / read-out parts of dg ------------------------------
template <int C>
__global__ void __launch_bounds__(NT, 1) bwd1_kernel(const __grid_constant__ CUtensorMap tm_qk,
                                                     const __grid_constant__ CUtensorMap tm_do,
                                                     const __grid_constant__ CUtensorMap tm_u,
                                                     const __grid_constant__ CUtensorMap tm_du,
                                                     const __grid_constant__ CUtensorMap tm_st,
                                                     const __grid_constant__ CUtensorMap tm_v, const Args a,
                                                     int v_col0) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  using S = BwdSmem;
  using WN = Win<C>;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + S::BARS);
  uint64_t* ld_bar = bars;
  uint64_t* mma_bar = bars + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2);
  const Meta m = carve_meta(sm + S::META);
  float* red = reinterpret_cast<float*>(sm + S::RED);
  float* inter = red + 4 * 128;          // [128] read-out decay term of the state part of each row
  const int r = threadIdx.x;
  const TileGeo t = tile_geo(a);
  constexpr int NCK = TR / C;
  if (r == 0) {
    mbar_init(ld_bar, 1);
    mbar_init(mma_bar, 1);
    fence_barrier_init();
  }
  if (r < 32) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t acc0 = tmem, acc1 = tmem + 128, acc2 = tmem + 256, acc3 = tmem + 384;
  const uint32_t sbase = smem_addr(sm);
  uint32_t mph = 0, lph = 0;
  bool ok = true;
  // S0 K | S1 dO -> dOg -> V -> Y | S2 U -> states -> dW^T | S3 dU | S4 A (fp32) -> dPE -> dT | S5 Q -> T
  if (r == 0) {
    mbar_expect_tx(ld_bar, 5 * TILE);
    load_rows(sm + S::S0, &tm_qk, ld_bar, 2 * t.hk + 1, t.t0, t.b);
    load_cols(sm + S::S1, &tm_do, ld_bar, t.hv * D, t.t0, t.b);
    load_rows(sm + S::S2, &tm_u, ld_bar, t.hv, t.t0, t.b);
    load_rows(sm + S::S3, &tm_du, ld_bar, t.hv, t.t0, t.b);
    load_rows(sm + S::S5, &tm_qk, ld_bar, 2 * t.hk, t.t0, t.b);
  }
  tile_meta<C>(a, t, m);
  WAIT_LD(231);
  const bool valid = t.p0 + r < t.Ls;
  const int cs = (r / C) * C;
  const int64_t grow0 = grow(a, t, 0);
  if (!valid) {
    // rows past the stream: no gradient flows in, and other streams' rows must not leak
#pragma unroll 1
    for (int g = 0; g < 4; ++g) {
      sm_zero32(sm + S::S1, r, g);
      sm_zero32(sm + S::S2, r, g);
      sm_zero32(sm + S::S3, r, g);
    }
  }
  SYNC_FOR_MMA();
  if (ok && r == 0) {
    tc_fence_after();
    mma(acc0, KM(sbase + S::S0), KM(sbase + S::S0), 128, 128, false);        // KK^T (kept to the end)
    mma(acc1, KM(sbase + S::S1), KM(sbase + S::S2), 128, 128, false);        // dP = dO U^T
    mma(acc3, KM(sbase + S::S5), KM(sbase + S::S0), 128, 128, false);        // QK^T
    umma_commit(mma_bar);
  }
  WAIT_MMA(232);
  float x[32], y[32];
  // A blocks (fp32, see af_idx) -> T (over Q, whose MMA is done)
  {
    float* Af = reinterpret_cast<float*>(sm + S::S4);
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
  invert_column<C>(reinterpret_cast<const float*>(sm + S::S4), sm + S::S5);
  __syncthreads();
  if (valid) {
    bf16* dst = a.tt + ((grow0 + r) * a.Hv + t.hv) * D;
#pragma unroll 1
    for (int g = 0; g < 4; ++g) {
      sm_ld32(sm + S::S5, r, g, x);
      gm_st32(dst + 32 * g, x);
    }
  }
  // dPE = dP . mask . e^{Gr_t - G_s} (tile + rows for bwd2); pair term dP . P of the decay gradient
  float dg = 0.f;
  {
    const float Gr = m.Gr[r];
    const int rd = m.rd[r], sg = m.seg[r];
    bf16* dst = a.dpe + ((grow0 + r) * a.Hv + t.hv) * D;
    PairSum<C> ps;
#pragma unroll 1
    for (int g = 0; g < 4; ++g) {
      if (g < WN::g0() || g >= WN::g0() + WN::NG) {
        sm_zero32(sm + S::S4, r, g);
#pragma unroll
        for (int i = 0; i < 32; ++i) x[i] = 0.f;
        if (valid) gm_st32(dst + 32 * g, x);
        continue;
      }
      tm_ld32(acc1, g, x);
      tm_ld32(acc3, g, y);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int s = 32 * g + i;
        const bool on = (s >= cs) && (s <= rd) && (m.seg[s] == sg) && valid;
        x[i] = on ? x[i] * __expf(Gr - m.G[s]) : 0.f;    // dPE
        y[i] = x[i] * y[i];                              // dP . P
      }
      sm_st32(sm + S::S4, r, g, x);
      if (valid) gm_st32(dst + 32 * g, x);
      ps.group(y, g, valid ? rd : -1, red);
    }
    __syncthreads();
    dg += PairSum<C>::total(red);
  }
  // dOg = carry e^{Gr} dO in place
  {
    const float qs = m.carry[r] * __expf(m.Gr[r]);
#pragma unroll 1
    for (int g = 0; g < 4; ++g) {
      sm_ld32(sm + S::S1, r, g, x);
      sm_st32(sm + S::S1, r, g, x, qs);
    }
  }
  SYNC_FOR_MMA();
  // dQ^T intra (acc2) = K^T dPE^T; per chunk: dQ^T inter (acc1) = S0 dOg^T, -dW^T (acc3) = S0 dU^T
  if (ok && r == 0) {
    tc_fence_after();
    mma(acc2, MN(sbase + S::S0), KM(sbase + S::S4), 128, 128, false);
    const int64_t sb = ((int64_t)t.b * a.Hv + t.hv) * a.nch;
    for (int c = 0; c < NCK && ok; ++c) {
      umma_commit(mma_bar);
      ok = mbar_wait(mma_bar, (mph + c) & 1, a.err, 233);   // S2 (U, then the previous state) is free
      if (!ok) break;
      int blk = t.p0 / C + c;
      blk = blk < a.nch ? blk : a.nch - 1;
      mbar_expect_tx(ld_bar, TILE);
      load_state(sm + S::S2, &tm_st, ld_bar, (int)((sb + blk) * D));
      ok = mbar_wait(ld_bar, (lph + c) & 1, a.err, 234);
      if (!ok) break;
      tc_fence_after();
      mma(acc1 + c * C, KM(sbase + S::S2), KM(sbase + S::S1, c * C), C, 128, false);
      mma(acc3 + c * C, KM(sbase + S::S2), KM(sbase + S::S3, c * C), C, 128, false);
    }
    umma_commit(mma_bar);
  }
  __syncthreads();
  mph += NCK;
  lph += NCK;
  WAIT_MMA(235);
  // dq rows = intra + inter (lanes k: transposed, coalesced per row); read-out decay term of the
  // state part: inter_t = q_t . dq_inter_t (a column dot over the 128 threads k)
  {
    const int nv = min(TR, t.Ls - t.p0);
    float* dst = a.dpart + grow0 * a.Hv * RED + t.hv * RED + r;
    const bf16* qcol = a.qk_rows + ((grow0 * a.Hk + t.hk) * 2) * D + r;   // q[t][k = r]
#pragma unroll 1
    for (int g = 0; g < 4; ++g) {
      tm_ld32(acc1, g, x);        // inter
      tm_ld32(acc2, g, y);        // intra
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int s = 32 * g + i;
        float qv = 0.f;
        if (s < nv) {
          dst[(int64_t)s * a.Hv * RED] = x[i] + y[i];
          qv = __bfloat162float(qcol[(int64_t)s * a.Hk * 2 * D]);
        }
        x[i] *= qv;
      }
      red[(r >> 5) * 128 + 32 * g + (r & 31)] = warp_colsum32(x);
    }
    __syncthreads();
    inter[r] = red[r] + red[128 + r] + red[256 + r] + red[384 + r];
    __syncthreads();
    // dg_j += sum of inter_t over rows t of j's segment that read out at or after j
    const int sg = m.seg[r];
    for (int tt = cs; tt < cs + C; ++tt)
      if (m.seg[tt] == sg && m.rd[tt] >= r) dg += inter[tt];
  }
  // dW^T (negated) into S2 as [k][t]; dW rows to global
  {
    bf16* dst = a.dw + grow0 * a.Hv * D + t.hv * D + r;
    const int nv = min(TR, t.Ls - t.p0);
#pragma unroll 1
    for (int g = 0; g < 4; ++g) {
      tm_ld32(acc3, g, x);
#pragma unroll
      for (int i = 0; i < 32; ++i) x[i] = -x[i];
      sm_st32(sm + S::S2, r, g, x);
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (32 * g + i < nv) dst[(int64_t)(32 * g + i) * a.Hv * D] = __float2bfloat16(x[i]);
    }
  }
  SYNC_FOR_MMA();
  // V into S1 (dOg is dead)
  if (ok && r == 0) {
    mbar_expect_tx(ld_bar, TILE);
    load_cols(sm + S::S1, &tm_v, ld_bar, v_col0 + t.hv * D, t.t0, t.b);
  }
  WAIT_LD(236);
  // dT: acc1 = dU V^T, acc2 = dW K^T  ->  dT_ts = beta_s (acc1 + carry_s e^{G_s} acc2), block diagonal
  if (ok && r == 0) {
    tc_fence_after();
    mma(acc1, KM(sbase + S::S3), KM(sbase + S::S1), 128, 128, false);
    mma(acc2, MN(sbase + S::S2), KM(sbase + S::S0), 128, 128, false);
    umma_commit(mma_bar);
  }
  WAIT_MMA(237);
#pragma unroll 1
  for (int g = 0; g < 4; ++g) {
    if (g < WN::g0() || g >= WN::g0() + WN::NG) {
      sm_zero32(sm + S::S4, r, g);    // dPE is dead (dQ done, rows saved)
      continue;
    }
    tm_ld32(acc1, g, x);
    tm_ld32(acc2, g, y);
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int s = 32 * g + i;
      const bool on = (s >= cs) && (s < cs + C);
      x[i] = on ? m.beta[s] * (x[i] + m.carry[s] * __expf(m.G[s]) * y[i]) : 0.f;
    }
    sm_st32(sm + S::S4, r, g, x);
  }
  SYNC_FOR_MMA();
  // Y = T^T dT (acc1), block diagonal
  if (ok && r == 0) {
    tc_fence_after();
    mma(acc1, MN(sbase + S::S5), MN(sbase + S::S4), 128, 128, false);
    umma_commit(mma_bar);
  }
  WAIT_MMA(238);
#pragma unroll 1
  for (int g = 0; g < 4; ++g) {
    if (g < WN::g0() || g >= WN::g0() + WN::NG) {
      sm_zero32(sm + S::S1, r, g);    // V is dead
      continue;
    }
    tm_ld32(acc1, g, x);
    sm_st32(sm + S::S1, r, g, x);
  }
  SYNC_FOR_MMA();
  // -dA = Y T^T (acc2)
  if (ok && r == 0) {
    tc_fence_after();
    mma(acc2, KM(sbase + S::S1), KM(sbase + S::S5), 128, 128, false);
    umma_commit(mma_bar);
  }
  WAIT_MMA(239);
  {
    const float Gt = m.G[r], bt = m.beta[r];
    const int sg = m.seg[r];
    float sa = 0.f;
    bf16* dst = a.dae + ((grow0 + r) * a.Hv + t.hv) * D;
    PairSum<C> ps;
#pragma unroll 1
    for (int g = 0; g < 4; ++g) {
      if (g < WN::g0() || g >= WN::g0() + WN::NG) {
#pragma unroll
        for (int i = 0; i < 32; ++i) x[i] = 0.f;
        if (valid) gm_st32(dst + 32 * g, x);
        continue;
      }
      tm_ld32(acc2, g, x);
      tm_ld32(acc0, g, y);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int s = 32 * g + i;
        const bool on = (s >= cs) && (s < r) && (m.seg[s] == sg) && valid;
        const float e = on ? __expf(Gt - m.G[s]) : 0.f;
        const float da = on ? -x[i] : 0.f;
        const float ke = y[i] * e;
        sa = fmaf(da, ke, sa);                    // d beta_t (A part)
        y[i] = da * bt * ke;                      // dA . A (pair term of the decay gradient)
        x[i] = da * bt * e;                       // dAE
      }
      if (valid) gm_st32(dst + 32 * g, x);
      ps.group(y, g, valid ? r : -1, red);
    }
    __syncthreads();
    dg += PairSum<C>::total(red);
    if (valid) {
      float* scp = a.sc + ((grow0 + r) * a.Hv + t.hv) * 2;
      scp[0] = sa;
      scp[1] = dg;
    }
  }
  tmem_wait_ld();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (r < 32) tmem_dealloc(tmem, 512);
}

// ---- bwd2: dV, dKb, dK, d beta, the one-sided parts of dg ------------------------------------------
template <int C>
__global__ void __launch_bounds__(NT, 1) bwd2_kernel(const __grid_constant__ CUtensorMap tm_qk,
                                                     const __grid_constant__ CUtensorMap tm_tt,
                                                     const __grid_constant__ CUtensorMap tm_du,
                                                     const __grid_constant__ CUtensorMap tm_dw,
                                                     const __grid_constant__ CUtensorMap tm_dpe,
                                                     const __grid_constant__ CUtensorMap tm_dae,
                                                     const __grid_constant__ CUtensorMap tm_u,
                                                     const __grid_constant__ CUtensorMap tm_st,
                                                     const __grid_constant__ CUtensorMap tm_dst, const Args a,
                                                     int v_col0) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  using S = BwdSmem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + S::BARS);
  uint64_t* ld_bar = bars;
  uint64_t* mma_bar = bars + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2);
  const Meta m = carve_meta(sm + S::META);
  float* red = reinterpret_cast<float*>(sm + S::RED);
  float* kb = red + 4 * 128;     // [128] dKb_t . Kb_t
  float* ksx = kb + 128;         // [128] k_s . (kts_s dS1 u_s) (clean stream)
  float* misc = ksx + 128;       // [4] warp partial sums
  const int r = threadIdx.x;
  const TileGeo t = tile_geo(a);
  constexpr int NCK = TR / C;
  if (r == 0) {
    mbar_init(ld_bar, 1);
    mbar_init(mma_bar, 1);
    fence_barrier_init();
  }
  if (r < 32) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t acc0 = tmem, acc1 = tmem + 128, acc2 = tmem + 256;
  const uint32_t sbase = smem_addr(sm);
  uint32_t mph = 0, lph = 0;
  bool ok = true;
  // S0 K | S1 T -> Q -> U | S2 dU -> dPE -> dS1 | S3 dW -> dAE -> S0
  if (r == 0) {
    mbar_expect_tx(ld_bar, 4 * TILE);
    load_rows(sm + S::S0, &tm_qk, ld_bar, 2 * t.hk + 1, t.t0, t.b);
    load_rows(sm + S::S1, &tm_tt, ld_bar, t.hv, t.t0, t.b);
    load_rows(sm + S::S2, &tm_du, ld_bar, t.hv, t.t0, t.b);
    load_rows(sm + S::S3, &tm_dw, ld_bar, t.hv, t.t0, t.b);
  }
  tile_meta<C>(a, t, m);
  const bool valid = t.p0 + r < t.Ls;
  const int cs = (r / C) * C;
  const int64_t row = grow(a, t, r), grow0 = grow(a, t, 0);
  float dbeta = 0.f, dg = 0.f;
  if (valid) {
    const float2 s1 = *reinterpret_cast<const float2*>(a.sc + (row * a.Hv + t.hv) * 2);
    dbeta = s1.x;
    dg = s1.y;
  }
  ksx[r] = 0.f;
  WAIT_LD(241);
  if (!valid) {
#pragma unroll 1
    for (int g = 0; g < 4; ++g) {
      sm_zero32(sm + S::S1, r, g);
      sm_zero32(sm + S::S2, r, g);
      sm_zero32(sm + S::S3, r, g);
    }
  }
  SYNC_FOR_MMA();
  if (ok && r == 0) {
    tc_fence_after();
    mma(acc0, MN(sbase + S::S1), MN(sbase + S::S2), 128, 128, false);   // dVb[s][v] = sum_t T[t][s] dU[t][v]
    mma(acc1, MN(sbase + S::S1), MN(sbase + S::S3), 128, 128, false);   // dKb[s][k] = sum_t T[t][s] dW[t][k]
    umma_commit(mma_bar);
  }
  WAIT_MMA(242);
  SYNC_FOR_MMA();
  if (ok && r == 0) {
    mbar_expect_tx(ld_bar, 3 * TILE);
    load_rows(sm + S::S1, &tm_qk, ld_bar, 2 * t.hk, t.t0, t.b);
    load_rows(sm + S::S2, &tm_dpe, ld_bar, t.hv, t.t0, t.b);
    load_rows(sm + S::S3, &tm_dae, ld_bar, t.hv, t.t0, t.b);
  }
  float x[32], y[32];
  const float ce = m.carry[r] * __expf(m.G[r]);
  const float ks = m.beta[r] * ce;
  // dV and the value part of d beta; the Kb parts of d beta and dg
  {
    const bf16* vrow = a.mixed + row * a.ldm + v_col0 + t.hv * D;
    bf16* dvrow = a.dv + row * a.lddv + t.hv * D;
    float kd = 0.f;
#pragma unroll 1
    for (int g = 0; g < 4; ++g) {
      tm_ld32(acc0, g, x);
      if (valid) {
        gm_st32(dvrow + 32 * g, x, m.beta[r]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint4 v = reinterpret_cast<const uint4*>(vrow + 32 * g)[j];
          const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
            dbeta = fmaf(f.x, x[8 * j + 2 * i], dbeta);
            dbeta = fmaf(f.y, x[8 * j + 2 * i + 1], dbeta);
          }
        }
      }
      tm_ld32(acc1, g, x);
      sm_ld32(sm + S::S0, r, g, y);
#pragma unroll
      for (int i = 0; i < 32; ++i) kd = fmaf(x[i], y[i], kd);
    }
    dbeta += ce * kd;
    kb[r] = valid ? ks * kd : 0.f;
  }
  WAIT_LD(243);
  if (!valid) {
#pragma unroll 1
    for (int g = 0; g < 4; ++g) {
      sm_zero32(sm + S::S2, r, g);
      sm_zero32(sm + S::S3, r, g);
    }
  }
  SYNC_FOR_MMA();
  if (ok && r == 0) {
    tc_fence_after();
    // dK (lanes s): dPE^T Q + dAE^T K (column parts) + dAE K (row part)
    mma(acc2, MN(sbase + S::S2), MN(sbase + S::S1), 128, 128, false);
    mma(acc2, MN(sbase + S::S3), MN(sbase + S::S0), 128, 128, true);
    mma(acc2, KM(sbase + S::S3), MN(sbase + S::S0), 128, 128, true);
    umma_commit(mma_bar);
  }
  WAIT_MMA(244);
  {
    float* dst = a.dpart + (row * a.Hv + t.hv) * RED + D;
#pragma unroll 1
    for (int g = 0; g < 4; ++g) {
      tm_ld32(acc2, g, x);
      tm_ld32(acc1, g, y);
      if (valid) {
#pragma unroll
        for (int i = 0; i < 32; i += 4)
          *reinterpret_cast<float4*>(dst + 32 * g + i) =
              make_float4(x[i] + ks * y[i], x[i + 1] + ks * y[i + 1], x[i + 2] + ks * y[i + 2], x[i + 3] + ks * y[i + 3]);
      }
    }
  }
  // end-state term of the clean chunks: dK_s += kts_s dS1 u_s; decay parts from k_s . (kts_s dS1 u_s)
  // and gamma <S0, dS1>
  float gsd = 0.f;   // gamma_c <S0_c, dS1_c> of this thread's chunk
  if (t.stream == 0) {
    SYNC_FOR_MMA();
    if (ok && r == 0) {
      mbar_expect_tx(ld_bar, TILE);
      load_rows(sm + S::S1, &tm_u, ld_bar, t.hv, t.t0, t.b);
    }
    WAIT_LD(245);
    {
      const float kt = valid ? m.kts[r] : 0.f;
#pragma unroll 1
      for (int g = 0; g < 4; ++g) {
        sm_ld32(sm + S::S1, r, g, x);
        sm_st32(sm + S::S1, r, g, x, kt);
      }
    }
    SYNC_FOR_MMA();
    const int64_t sb = ((int64_t)t.b * a.Hv + t.hv) * a.nch;
    for (int c = 0; c < NCK; ++c) {
      int blk = t.p0 / C + c;
      const bool real = blk < a.nch;
      blk = real ? blk : a.nch - 1;
      if (ok && r == 0) {
        mbar_expect_tx(ld_bar, 2 * TILE);
        load_state(sm + S::S2, &tm_dst, ld_bar, (int)((sb + blk) * D));
        load_state(sm + S::S3, &tm_st, ld_bar, (int)((sb + blk) * D));
      }
      WAIT_LD(246);
      if (ok && r == 0) {
        tc_fence_after();
        mma(acc0 + c * C, KM(sbase + S::S2), KM(sbase + S::S1, c * C), C, 128, false);
        umma_commit(mma_bar);
      }
      {
        float d = 0.f;
#pragma unroll 1
        for (int g = 0; g < 4; ++g) {
          sm_ld32(sm + S::S3, r, g, x);
          sm_ld32(sm + S::S2, r, g, y);
#pragma unroll
          for (int i = 0; i < 32; ++i) d = fmaf(x[i], y[i], d);
        }
        d = warp_sum(d);
        if ((r & 31) == 0) misc[r >> 5] = d;
      }
      WAIT_MMA(247);
      __syncthreads();
      if (r / C == c && real) gsd = a.gamma[sb + blk] * (misc[0] + misc[1] + misc[2] + misc[3]);
      SYNC_FOR_MMA();   // S2 / S3 are reloaded next chunk; misc is rewritten
    }
    // X^T[k][s] (lanes k): ksx_s = sum_k X^T[k][s] K[s][k]; dk rows += X^T (transposed)
    {
      float* dst = a.dpart + grow0 * a.Hv * RED + t.hv * RED + D + r;
      const int nv = min(TR, t.Ls - t.p0);
#pragma unroll 1
      for (int g = 0; g < 4; ++g) {
        tm_ld32(acc0, g, x);
#pragma unroll
        for (int i = 0; i < 32; ++i) y[i] = x[i] * ld_el(sm + S::S0, 32 * g + i, r);
        red[(r >> 5) * 128 + 32 * g + (r & 31)] = warp_colsum32(y);
      }
      __syncthreads();   // every dk row above is written (and the partial sums)
      ksx[r] = red[r] + red[128 + r] + red[256 + r] + red[384 + r];
#pragma unroll 1
      for (int g = 0; g < 4; ++g) {
        tm_ld32(acc0, g, x);
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (32 * g + i < nv) dst[(int64_t)(32 * g + i) * a.Hv * RED] += x[i];
      }
    }
  }
  __syncthreads();
  // one-sided decay terms: Kb rows at or after j in j's segment; K~ rows before j and gamma when j
  // lies in the chunk's last segment
  if (valid) {
    const int sg = m.seg[r], last = cs + C - 1;
    for (int tt = r; tt < cs + C && m.seg[tt] == sg; ++tt) dg += kb[tt];
    if (sg == m.seg[last]) {
      for (int s = cs; s < r; ++s)
        if (m.seg[s] == sg) dg += ksx[s];
      dg += gsd;
    }
    float* dst = a.dpart + (row * a.Hv + t.hv) * RED + 2 * D;
    dst[0] = dbeta;
    dst[1] = dg;
  }
  tmem_wait_ld();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (r < 32) tmem_dealloc(tmem, 512);
}

// ---- post: sum the value heads of each key head, q/k L2-norm backward, gate backward -------------------
__global__ void post_kernel(const Args a, const bf16* ga, const bf16* gbeta, int64_t ldg, const float* A_log,
                            const float* dt_bias, float scale, bf16* dmixed, int64_t lddm, bf16* dga, bf16* dgb,
                            int64_t lddg, float* dA_log, float* ddt_bias) {
  const int64_t row = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const int rep = a.Hv / a.Hk;
  const bf16* src = a.mixed + row * a.ldm;
  for (int w = warp; w < 2 * a.Hk; w += nw) {
    const int hk = w >> 1, isk = w & 1;
    float xv[4], g[4] = {0.f, 0.f, 0.f, 0.f};
    const bf16* xp = src + isk * a.Hk * D + hk * D + lane * 4;
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      xv[e] = __bfloat162float(xp[e]);
      ss += xv[e] * xv[e];
    }
    for (int rr = 0; rr < rep; ++rr) {
      const float4 d = *reinterpret_cast<const float4*>(a.dpart + (row * a.Hv + hk * rep + rr) * RED + isk * D + lane * 4);
      g[0] += d.x; g[1] += d.y; g[2] += d.z; g[3] += d.w;
    }
    ss = warp_sum(ss);
    const float rn = rsqrtf(ss + 1e-6f);
    const float sc = isk ? 1.f : scale;
    float dot = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      g[e] *= sc;
      dot += xv[e] * rn * g[e];
    }
    dot = warp_sum(dot);
    bf16* dp = dmixed + row * lddm + isk * a.Hk * D + hk * D + lane * 4;
#pragma unroll
    for (int e = 0; e < 4; ++e) dp[e] = __float2bfloat16(rn * (g[e] - xv[e] * rn * dot));
  }
  for (int h = threadIdx.x; h < a.Hv; h += blockDim.x) {
    const float* pr = a.dpart + (row * a.Hv + h) * RED + 2 * D;
    const float dbeta = pr[0], dg = pr[1];
    const float xa = __bfloat162float(ga[row * ldg + h]) + dt_bias[h];
    const float bv = __bfloat162float(gbeta[row * ldg + h]);
    const float beta = 1.f / (1.f + expf(-bv));
    const float eA = expf(A_log[h]);
    const float sp = xa > 20.f ? xa : log1pf(expf(xa));
    const float sig = xa > 20.f ? 1.f : 1.f / (1.f + expf(-xa));
    const float da = dg * (-eA) * sig;
    dga[row * lddg + h] = __float2bfloat16(da);
    dgb[row * lddg + h] = __float2bfloat16(dbeta * beta * (1.f - beta));
    atomicAdd(dA_log + h, dg * (-eA * sp));
    atomicAdd(ddt_bias + h, da);
  }
}

template <int C>
static int launch_bwd(const GdnChunkBwdParams& p, const Args& a, cudaStream_t st) {
  const GdnChunkParams& f = p.fwd;
  CUtensorMap m_qk, m_do, m_u, m_du, m_st, m_dst, m_v, m_tt, m_dw, m_dpe, m_dae, m_ds0;
  CUtensorMap c_kt, c_qg, c_do, c_wn, c_du0, c_qk, c_du;
  if (!map_heads(&m_qk, f.qk, f.B, f.T, 2 * f.Hk, TR)) return -2;
  if (!map_cols(&m_do, p.d_o, f.B, f.T, (int64_t)f.Hv * D, (int64_t)f.Hv * D, TR)) return -3;
  if (!map_heads(&m_u, f.u, f.B, f.T, f.Hv, TR)) return -4;
  if (!map_heads(&m_du, p.du, f.B, f.T, f.Hv, TR)) return -5;
  if (!map_cols(&m_st, f.ckpt, 1, f.B * f.Hv * f.nch * D, D, D, 128)) return -6;
  if (!map_cols(&m_dst, p.dckpt, 1, f.B * f.Hv * f.nch * D, D, D, 128)) return -7;
  if (!map_cols(&m_v, f.mixed, f.B, f.T, 2 * f.Hk * D + f.Hv * D, f.ldm, TR)) return -8;
  if (!map_heads(&m_tt, p.tt, f.B, f.T, f.Hv, TR)) return -9;
  if (!map_heads(&m_dw, p.dw, f.B, f.T, f.Hv, TR)) return -10;
  if (!map_heads(&m_dpe, p.dpe, f.B, f.T, f.Hv, TR)) return -11;
  if (!map_heads(&m_dae, p.dae, f.B, f.T, f.Hv, TR)) return -12;
  if (!map_cols(&m_ds0, p.ds0, 1, f.B * f.Hv * f.nch * D, D, D, 128)) return -13;
  if (!map_heads(&c_kt, f.kt, f.B, f.T, f.Hv, C)) return -14;
  if (!map_heads(&c_qg, p.qg, f.B, f.T, f.Hv, C)) return -15;
  if (!map_cols(&c_do, p.d_o, f.B, f.T, (int64_t)f.Hv * D, (int64_t)f.Hv * D, C)) return -16;
  if (!map_heads(&c_wn, f.wn, f.B, f.T, f.Hv, C)) return -17;
  if (!map_heads(&c_du0, p.du0, f.B, f.T, f.Hv, C)) return -18;
  if (!map_heads(&c_qk, f.qk, f.B, f.T, 2 * f.Hk, C)) return -19;
  if (!map_heads(&c_du, p.du, f.B, f.T, f.Hv, C)) return -20;
  const int v_col0 = 2 * f.Hk * D;
  const int bsmem = BwdSmem::TOTAL + 1024;
  const int dsmem = 4 * C * 256 + 64 + 4 * C + 1024 + 64;
  const int csmem = ScanbSmem<C, false>::TOTAL + 1024, nsmem = ScanbSmem<C, true>::TOTAL + 1024;
  static bool init = false;
  if (!init) {
    cudaFuncSetAttribute(bwd0_kernel<C>, cudaFuncAttributeMaxDynamicSharedMemorySize, bsmem);
    cudaFuncSetAttribute(bwd1_kernel<C>, cudaFuncAttributeMaxDynamicSharedMemorySize, bsmem);
    cudaFuncSetAttribute(bwd2_kernel<C>, cudaFuncAttributeMaxDynamicSharedMemorySize, bsmem);
    cudaFuncSetAttribute(ds0_kernel<C>, cudaFuncAttributeMaxDynamicSharedMemorySize, dsmem);
    cudaFuncSetAttribute(scanb_kernel<C, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, csmem);
    cudaFuncSetAttribute(scanb_kernel<C, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, nsmem);
    init = true;
  }
  const int Lc = f.mode ? f.L : f.T;
  const int tiles = (Lc + TR - 1) / TR;
  const int ns = f.mode ? 1 + f.V : 1;
  bwd0_kernel<C><<<dim3(tiles, f.Hv, f.B * ns), NT, bsmem, st>>>(m_qk, m_do, a);
  if (f.mode) {
    ds0_kernel<C><<<dim3(f.nch, f.Hv, f.B), NT, dsmem, st>>>(c_qk, c_do, c_wn, c_du, a);
    scanb_kernel<C, true><<<dim3(f.Hv, f.B), NT, nsmem, st>>>(c_kt, c_qg, c_do, c_wn, c_du0, m_ds0, a);
  } else {
    scanb_kernel<C, false><<<dim3(f.Hv, f.B), NT, csmem, st>>>(c_kt, c_qg, c_do, c_wn, c_du0, m_ds0, a);
  }
  bwd1_kernel<C><<<dim3(tiles, f.Hv, f.B * ns), NT, bsmem, st>>>(m_qk, m_do, m_u, m_du, m_st, m_v, a, v_col0);
  bwd2_kernel<C><<<dim3(tiles, f.Hv, f.B * ns), NT, bsmem, st>>>(m_qk, m_tt, m_du, m_dw, m_dpe, m_dae, m_u, m_st,
                                                                   m_dst, a, v_col0);
  post_kernel<<<f.B * f.T, 256, 0, st>>>(a, f.ga, f.gbeta, f.ldg, f.A_log, f.dt_bias, f.scale, p.dmixed, p.lddm, p.dga,
                                         p.dgb, p.lddg, p.dA_log, p.ddt_bias);
  return 0;
}

}  // namespace gdnc

using namespace gdnc;

int gdn_chunk_bwd(const GdnChunkBwdParams& p, cudaStream_t st) {
  const GdnChunkParams& f = p.fwd;
  Args a{};
  a.B = f.B; a.T = f.T; a.Hk = f.Hk; a.Hv = f.Hv; a.mode = f.mode; a.L = f.L; a.V = f.V;
  a.nch = f.nch; a.tok_clean = f.causal_clean; a.tok_noisy = f.causal_noisy; a.doc = f.doc; a.gb = f.gb;
  a.o = nullptr; a.ckpt = f.ckpt; a.gamma = f.gamma; a.final_state = nullptr;
  a.wn = f.wn; a.ut = f.ut; a.kt = f.kt; a.u = f.u; a.err = f.err;
  a.o_fwd = f.o; a.d_o = p.d_o; a.du0 = p.du0; a.du = p.du; a.qg = p.qg; a.ds0 = p.ds0; a.dckpt = p.dckpt;
  a.dpe = p.dpe; a.dae = p.dae; a.dw = p.dw; a.tt = p.tt; a.sc = p.sc; a.dpart = p.dpart;
  a.dv = p.dmixed + 2 * f.Hk * D; a.lddv = p.lddm;
  a.mixed = f.mixed; a.ldm = f.ldm; a.qk_rows = f.qk;
  int rc;
  switch (f.C) {
    case 16: rc = launch_bwd<16>(p, a, st); break;
    case 32: rc = launch_bwd<32>(p, a, st); break;
    case 64: rc = launch_bwd<64>(p, a, st); break;
    default: return -1;
  }
  if (rc != 0) return rc;
  return cudaGetLastError() == cudaSuccess ? 0 : -30;
}

}  // namespace trida
