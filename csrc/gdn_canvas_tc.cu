// Serving canvas step of the gated-delta layers on the 5th-generation tensor cores.
//
// A decode canvas of n <= 64 rows of one request starts from the slot's state S0 [dk = 128, dv =
// 128] (fp32).  Rows t < n_clean read out the state after their own row, the other rows the state
// after the whole canvas (the block-causal draft rows of self-speculative decoding):
//     S_t = a_t S_{t-1} + k_t u_t^T,   u_t = b_t (v_t - a_t S_{t-1}^T k_t),   o_t = S_{r(t)}^T q_t,
// with r(t) = t for t < n_clean and n - 1 otherwise (q, k L2-normalised, q scaled by dk^-1/2).  One
// canvas is exactly one chunk of the chunked (WY) form; with G_t = sum_{s<=t} log a_s:
//     A_ts = b_t e^{G_t - G_s} k_t.k_s (s < t),   T = (I + A)^-1
//     W = T diag(b e^G) K,   U = T diag(b) V - W S0
//     O = diag(e^{G_r}) Q S0 + P U,   P_ts = q_t.k_s e^{G_{r(t)} - G_s} (s <= r(t))
// and the state after the first m rows (the commit of m accepted rows) is
//     S_m = e^{G_{m-1}} S0 + sum_{s<m} e^{G_{m-1} - G_s} k_s u_s^T.
// So the canvas kernel stores each row's normalised k, its U row and G, and the commit is one
// [dk x m] x [m x dv] product plus the decayed old state -- the accepted rows are not re-run.
//
// canvas_kernel: CTA = (value head, request), 128 threads, thread t = tile row t = TMEM lane t.
// Operands are bf16 tiles of 64 rows ([64][64] 128-byte swizzled halves, 8 KB each) except S0
// ([128][128], 32 KB).  Every product is an M = 128 tcgen05.mma: rows 64..127 of the A operand
// read the bytes that follow the tile (finite data of the next tile), which only produces
// accumulator rows 64..127 that nobody reads; contractions over canvas rows use K = 64 so the B
// operand is read only in its 64 real rows.  About 105 KB of shared memory and 256 TMEM columns per
// CTA, so two CTAs share an SM.  Phases (thread 0 issues, every thread waits on one mbarrier):
//   1  KK = K K^T, QK = Q K^T                   -> TMEM [0,64), [64,128)
//      rows: A (fp32, shared memory), Kb = diag(b e^G) K over K, Qg = diag(e^{G_r}) Q over Q
//      columns: T = (I + A)^-1 by forward substitution; rows: P from QK over A
//   2  W = T Kb, U~ = T Vb                       -> TMEM [0,128), [128,256)
//      rows: -W over Vb
//   3  U = U~ + (-W) S0                          -> TMEM [128,256)
//      rows: U over -W (and to global for the commit)
//   4  O = Qg S0 + P U                           -> TMEM [0,128); rows: O to global
// commit_kernel: CTA = (value head, request): K~ rows k_s e^{G_{m-1} - G_s} (s < m) and U rows as
// [64][128] tiles, S_m = K~^T U in TMEM (M = dk), plus e^{G_{m-1}} S0 while the rows are written.
// Every mbarrier wait is bounded (error word), no TMA and no multicast.
#include "gdn_chunk.cuh"

namespace trida {
namespace gdncv {

using namespace trida::sm100;
using gdnc::af_idx;
using gdnc::KM;
using gdnc::MN;
using gdnc::mma;
using gdnc::pack_bf2;

constexpr int NT = 128;
constexpr int C = 64;                  // rows of a canvas tile
constexpr int H64 = 64 * 128;          // bytes of one [64][64] bf16 half
constexpr int T64 = 2 * H64;           // a [64][128] bf16 tile
constexpr int S128 = 128 * 128;        // one [128][64] half of the S0 tile

// byte offset of (row, col) in a [64][128] tile (two 64-column halves)
__device__ __forceinline__ uint32_t off64(int r, int c) { return (uint32_t)(c >> 6) * H64 + sw128_offset(r, c & 63); }
__device__ __forceinline__ uint32_t off128(int r, int c) { return (uint32_t)(c >> 6) * S128 + sw128_offset(r, c & 63); }

struct CanvasSmem {
  static constexpr int RQ = 0;             // Q -> Qg
  static constexpr int RK = RQ + T64;      // K -> Kb
  static constexpr int RV = RK + T64;      // Vb -> -W -> U
  static constexpr int RA = RV + T64;      // A (fp32 64 x 64) -> P ([64][64] bf16)
  static constexpr int RT = RA + T64;      // T ([64][64] bf16)
  static constexpr int RS = RT + H64;      // S0 ([128][128] bf16)
  static constexpr int META = RS + 2 * S128;
  static constexpr int BAR = META + 4 * 64 * 4;
  static constexpr int TOTAL = BAR + 64;
};

struct CanvasArgs {
  const bf16* mixed; int64_t ldm;        // [B * n, ldm]: q | k (Hk heads of 128), v (Hv heads of 128)
  const bf16* ga; const bf16* gb; int64_t ldg;   // [B * n, ldg] decay input / beta logit per value head
  const float* A_log; const float* dt_bias;      // [Hv]
  const float* ssm;                      // [slots, Hv, 128, 128] fp32 (k rows, v columns)
  const int* slot;                       // [B]
  bf16* o;                               // [B * n, Hv * 128]: o, or y = rmsnorm(o) * w * silu(z) when
  const bf16* z; int64_t ldz;            //   z (gate rows [B * n, ldz], value head h at column 128 h)
  const bf16* gnorm_w; float eps;        //   and the norm weight [128] are given
  bf16* kbuf; bf16* ubuf;                // [B * n, Hv, 128] normalised k / U rows (commit inputs)
  float* gbuf;                           // [B * n, Hv] cumulative log decay G
  int* err;
  int n, n_clean, Hk, Hv;
  float scale;
};

__device__ __forceinline__ float softplus_(float x) { return x > 20.f ? x : log1pf(expf(x)); }

// 16-byte load of 8 bf16 as fp32
__device__ __forceinline__ void ld8(const bf16* p, float (&f)[8]) {
  const uint4 v = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 x = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
    f[2 * i] = x.x;
    f[2 * i + 1] = x.y;
  }
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}

// sum of squares of bf16 row r of a [64][128] tile
__device__ __forceinline__ float rowsq(const uint8_t* tile, int r) {
  float s2 = 0.f;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const uint4 v = *reinterpret_cast<const uint4*>(tile + off64(r, 8 * j));
    const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w4[i]));
      s2 = fmaf(f.x, f.x, fmaf(f.y, f.y, s2));
    }
  }
  return s2;
}

// row r of a [64][128] tile times `mul`, in place (and to `gdst` when given)
__device__ __forceinline__ void scale_row(uint8_t* tile, int r, float mul, bf16* gdst) {
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    uint4* p = reinterpret_cast<uint4*>(tile + off64(r, 8 * j));
    const uint4 v = *p;
    const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
    uint32_t o4[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w4[i]));
      o4[i] = pack_bf2(f.x * mul, f.y * mul);
    }
    const uint4 o = make_uint4(o4[0], o4[1], o4[2], o4[3]);
    *p = o;
    if (gdst) reinterpret_cast<uint4*>(gdst)[j] = o;
  }
}

// 16 vectors of 8 bf16 (one 128-element row), times `mul`, as bf16 row r of a [64][128] tile (and to
// `gdst` when given)
__device__ __forceinline__ void store_row(const uint4 (&x)[16], float mul, uint8_t* tile, int r, bf16* gdst) {
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const uint32_t w4[4] = {x[j].x, x[j].y, x[j].z, x[j].w};
    uint32_t o4[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w4[i]));
      o4[i] = pack_bf2(f.x * mul, f.y * mul);
    }
    const uint4 v = make_uint4(o4[0], o4[1], o4[2], o4[3]);
    *reinterpret_cast<uint4*>(tile + off64(r, 8 * j)) = v;
    if (gdst) reinterpret_cast<uint4*>(gdst)[j] = v;
  }
}

__device__ __forceinline__ void zero_row(uint8_t* tile, int r, int cols) {
  const uint4 z = make_uint4(0, 0, 0, 0);
  for (int j = 0; j < cols / 8; ++j) *reinterpret_cast<uint4*>(tile + off64(r, 8 * j)) = z;
}

// 32 fp32 TMEM columns of this thread's lane
__device__ __forceinline__ void tld32(uint32_t taddr, float (&x)[32]) {
  uint32_t v[32];
  tmem_ld32(taddr + ((uint32_t)(32 * (threadIdx.x >> 5)) << 16), v);
  tmem_wait_ld();
#pragma unroll
  for (int i = 0; i < 32; ++i) x[i] = __uint_as_float(v[i]);
}

// issue-and-wait step: every thread arrives here after its shared-memory writes
struct Phase {
  uint64_t* bar;
  int* err;
  uint32_t n = 0;
  __device__ bool wait() {
    const bool ok = mbar_wait(bar, n & 1, err, 80 + (int)n);
    ++n;
    tc_fence_after();
    return ok;
  }
};

__global__ void __launch_bounds__(NT) canvas_kernel(const CanvasArgs a) {
  using S = CanvasSmem;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  float* G = reinterpret_cast<float*>(smem + S::META);       // [64] cumulative log decay
  float* be = G + 64;                                         // [64] beta
  float* gl = G + 128;                                        // [64] log decay
  float* Gr = G + 192;                                        // [64] G at the read-out row
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + S::BAR);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + S::BAR + 8);
  uint8_t *tQ = smem + S::RQ, *tK = smem + S::RK, *tV = smem + S::RV, *tA = smem + S::RA, *tT = smem + S::RT,
          *tS = smem + S::RS;
  float* Af = reinterpret_cast<float*>(tA);
  const int hv = blockIdx.x, b = blockIdx.y, t = threadIdx.x, w = t >> 5;
  const int n = a.n, hk = hv / (a.Hv / a.Hk), kd = a.Hk * 128;
  const int64_t row = (int64_t)b * n + t;
  const bool live = t < n;

  if (t == 0) {
    mbar_init(bar, 1);
    fence_barrier_init();
  }
  if (w == 0) tmem_alloc(tslot, 256);
  // ---- rows: the q / k / v rows land in their tile positions by cp.async (3 x 64 rows x 16 copies of
  //      16 bytes, all in flight at once); rows past the canvas are zero.  Then, in shared memory,
  //      q / k are L2-normalised (q times the scale) and v is scaled by beta ----
  for (int it = t; it < 3 * C * 16; it += NT) {
    const int kind = it / (C * 16), rem = it % (C * 16), r = rem >> 4, j = rem & 15;
    uint8_t* dst = (kind == 0 ? tQ : kind == 1 ? tK : tV) + off64(r, 8 * j);
    if (r < n) {
      const int64_t col = kind == 0 ? hk * 128 : kind == 1 ? kd + hk * 128 : 2 * kd + hv * 128;
      cp_async16(dst, a.mixed + ((int64_t)b * n + r) * a.ldm + col + 8 * j);
    } else {
      *reinterpret_cast<uint4*>(dst) = make_uint4(0u, 0u, 0u, 0u);
    }
  }
  asm volatile("cp.async.commit_group;\n" ::: "memory");
  if (t < C) {
    if (live) {
      const float av = __bfloat162float(a.ga[row * a.ldg + hv]) + a.dt_bias[hv];
      const float bv = __bfloat162float(a.gb[row * a.ldg + hv]);
      gl[t] = -expf(a.A_log[hv]) * softplus_(av);
      be[t] = 1.f / (1.f + expf(-bv));
    } else {
      gl[t] = 0.f;
      be[t] = 0.f;
    }
  }
  {  // S0 row t (k index t) as bf16: two batches of 16 vector loads
    const float* src = a.ssm + (((int64_t)a.slot[b] * a.Hv + hv) * 128 + t) * 128;
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
      float4 x[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) x[j] = reinterpret_cast<const float4*>(src)[16 * h2 + j];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        *reinterpret_cast<uint4*>(tS + off128(t, 64 * h2 + 8 * j)) =
            make_uint4(pack_bf2(x[2 * j].x, x[2 * j].y), pack_bf2(x[2 * j].z, x[2 * j].w),
                       pack_bf2(x[2 * j + 1].x, x[2 * j + 1].y), pack_bf2(x[2 * j + 1].z, x[2 * j + 1].w));
    }
  }
  asm volatile("cp.async.wait_all;\n" ::: "memory");
  __syncthreads();
  // threads 0-63: q row t (norm, times the scale), then v row t (times beta); threads 64-127: k row
  // t - 64 (norm; also to kbuf for the commit)
  {
    const int r = t & (C - 1);
    if (r < n) {
      uint8_t* tile = t < C ? tQ : tK;
      const float ss = rowsq(tile, r);
      const float mul = rsqrtf(ss + 1e-6f) * (t < C ? a.scale : 1.f);
      scale_row(tile, r, mul, t < C ? nullptr : a.kbuf + (((int64_t)b * n + r) * a.Hv + hv) * 128);
      if (t < C) scale_row(tV, r, be[r], nullptr);
    }
  }
  if (t < C) {
    float s = 0.f;
    for (int j = 0; j <= t; ++j) s += gl[j];
    G[t] = s;
  }
  __syncthreads();
  const int rt = t < a.n_clean ? t : n - 1;             // read-out row
  float Gt = 0.f, Grt = 0.f, bt = 0.f;
  if (t < C) {
    Gt = G[t];
    Grt = G[rt < 0 ? 0 : rt];
    bt = be[t];
    Gr[t] = Grt;
    if (live) a.gbuf[row * a.Hv + hv] = Gt;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  Phase ph{bar, a.err};
  bool ok = true;
  // ---- phase 1: KK = K K^T, QK = Q K^T (64 key columns each) ----
  fence_async_smem();
  __syncthreads();
  if (t == 0) {
    tc_fence_after();
    mma(tmem, KM(smem_addr(tK), 0, 0, H64), KM(smem_addr(tK), 0, 0, H64), 64, 128, false);
    mma(tmem + 64, KM(smem_addr(tQ), 0, 0, H64), KM(smem_addr(tK), 0, 0, H64), 64, 128, false);
    umma_commit(bar);
  }
  ok = ph.wait();
  if (w < 2) {
    // A row t (fp32, chunk-local columns) and the scaled Q / K rows for the next products
    float x[32];
#pragma unroll 1
    for (int g2 = 0; g2 < 2; ++g2) {
      tld32(tmem + 32 * g2, x);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int s = 32 * g2 + i;
        Af[af_idx(t, s)] = (s < t && live) ? bt * __expf(Gt - G[s]) * x[i] : 0.f;
      }
    }
  }
  __syncthreads();                     // A complete; Q / K rows are read below, then rewritten
  if (t < C) {
    // Kb = diag(b e^G) K over K, Qg = diag(e^{G_r}) Q over Q (their MMAs of phase 1 have run)
    const float kb = live ? bt * __expf(Gt) : 0.f, qg = live ? __expf(Grt) : 0.f;
#pragma unroll 4
    for (int j = 0; j < 16; ++j) {
      uint4* pk = reinterpret_cast<uint4*>(tK + off64(t, 8 * j));
      uint4* pq = reinterpret_cast<uint4*>(tQ + off64(t, 8 * j));
      uint4 vk = *pk, vq = *pq;
      uint32_t* ek = reinterpret_cast<uint32_t*>(&vk);
      uint32_t* eq = reinterpret_cast<uint32_t*>(&vq);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 fk = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ek[i]));
        const float2 fq = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&eq[i]));
        ek[i] = pack_bf2(fk.x * kb, fk.y * kb);
        eq[i] = pack_bf2(fq.x * qg, fq.y * qg);
      }
      *pk = vk;
      *pq = vq;
    }
    // column t of T = (I + A)^-1 by forward substitution
    float xs[C];
#pragma unroll
    for (int i = 0; i < C; ++i) xs[i] = (i == t) ? 1.f : 0.f;
#pragma unroll
    for (int i = 1; i < C; ++i) {
      float s4[4] = {0.f, 0.f, 0.f, 0.f};     // four independent chains instead of one of length i
#pragma unroll
      for (int u = 0; u < i; ++u) s4[u & 3] = fmaf(Af[af_idx(i, u)], xs[u], s4[u & 3]);
      if (i > t) xs[i] = -((s4[0] + s4[1]) + (s4[2] + s4[3]));
    }
#pragma unroll
    for (int i = 0; i < C; ++i) *reinterpret_cast<bf16*>(tT + sw128_offset(i, t)) = __float2bfloat16(xs[i]);
  }
  __syncthreads();                     // every column of T is written, A is no longer read
  if (w < 2) {
    // P row t over A: q_t.k_s e^{G_r(t) - G_s} for s <= r(t), bf16 [64][64]
    float x[32];
#pragma unroll 1
    for (int g2 = 0; g2 < 2; ++g2) {
      tld32(tmem + 64 + 32 * g2, x);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float f[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int s = 32 * g2 + 8 * j + i;
          f[i] = (live && s <= rt && s < n) ? x[8 * j + i] * __expf(Grt - G[s]) : 0.f;
        }
        *reinterpret_cast<uint4*>(tA + sw128_offset(t, 32 * g2 + 8 * j)) =
            make_uint4(pack_bf2(f[0], f[1]), pack_bf2(f[2], f[3]), pack_bf2(f[4], f[5]), pack_bf2(f[6], f[7]));
      }
    }
  }
  // ---- phase 2: W = T Kb, U~ = T Vb ----
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  if (t == 0) {
    tc_fence_after();
    mma(tmem, KM(smem_addr(tT), 0, 0, H64), MN(smem_addr(tK), 0, H64), 128, C, false);
    mma(tmem + 128, KM(smem_addr(tT), 0, 0, H64), MN(smem_addr(tV), 0, H64), 128, C, false);
    umma_commit(bar);
  }
  ok = ph.wait() && ok;
  if (a.z != nullptr) {                // the fused norm's gate rows into the K tile (free once phase 2 ran),
    for (int it = t; it < C * 16; it += NT) {      // in flight under phases 3 and 4
      const int r = it >> 4, j = it & 15;
      if (r < n) cp_async16(tK + off64(r, 8 * j), a.z + ((int64_t)b * n + r) * a.ldz + hv * 128 + 8 * j);
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
  }
  if (w < 2) {                         // -W over Vb (the U~ product has read it)
    float x[32];
#pragma unroll 1
    for (int g4 = 0; g4 < 4; ++g4) {
      tld32(tmem + 32 * g4, x);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        *reinterpret_cast<uint4*>(tV + off64(t, 32 * g4 + 8 * j)) =
            make_uint4(pack_bf2(-x[8 * j], -x[8 * j + 1]), pack_bf2(-x[8 * j + 2], -x[8 * j + 3]),
                       pack_bf2(-x[8 * j + 4], -x[8 * j + 5]), pack_bf2(-x[8 * j + 6], -x[8 * j + 7]));
    }
  }
  // ---- phase 3: U = U~ + (-W) S0 ----
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  if (t == 0) {
    tc_fence_after();
    mma(tmem + 128, KM(smem_addr(tV), 0, 0, H64), MN(smem_addr(tS), 0, S128), 128, 128, true);
    umma_commit(bar);
  }
  ok = ph.wait() && ok;
  if (w < 2) {                         // U over -W, and the U row to global for the commit
    float x[32];
    bf16* gu = a.ubuf + (row * a.Hv + hv) * 128;
#pragma unroll 1
    for (int g4 = 0; g4 < 4; ++g4) {
      tld32(tmem + 128 + 32 * g4, x);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 v = make_uint4(pack_bf2(x[8 * j], x[8 * j + 1]), pack_bf2(x[8 * j + 2], x[8 * j + 3]),
                                   pack_bf2(x[8 * j + 4], x[8 * j + 5]), pack_bf2(x[8 * j + 6], x[8 * j + 7]));
        *reinterpret_cast<uint4*>(tV + off64(t, 32 * g4 + 8 * j)) = v;
        if (live) reinterpret_cast<uint4*>(gu)[4 * g4 + j] = v;
      }
    }
  }
  // ---- phase 4: O = Qg S0 + P U ----
  asm volatile("cp.async.wait_all;\n" ::: "memory");
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  if (t == 0) {
    tc_fence_after();
    mma(tmem, KM(smem_addr(tQ), 0, 0, H64), MN(smem_addr(tS), 0, S128), 128, 128, false);
    mma(tmem, KM(smem_addr(tA), 0, 0, H64), MN(smem_addr(tV), 0, H64), 128, C, true);
    umma_commit(bar);
  }
  ok = ph.wait() && ok;
  if (w < 2) {                         // tcgen05.ld is warp-collective: every lane loads, live rows store
    float x[32];
    bf16* go = a.o + row * (int64_t)(a.Hv * 128) + hv * 128;
    float rs = 1.f;
    if (a.z != nullptr) {              // gated RMSNorm of this head's row: first its mean square
      float ss = 0.f;
#pragma unroll 1
      for (int g4 = 0; g4 < 4; ++g4) {
        tld32(tmem + 32 * g4, x);
#pragma unroll
        for (int i = 0; i < 32; ++i) ss = fmaf(x[i], x[i], ss);
      }
      rs = rsqrtf(ss * (1.f / 128.f) + a.eps);
    }
#pragma unroll 1
    for (int g4 = 0; g4 < 4; ++g4) {
      tld32(tmem + 32 * g4, x);
      if (a.z != nullptr && live) {
        const bf16* wr = a.gnorm_w + 32 * g4;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float zf[8], wf[8];
          const uint4 zv = *reinterpret_cast<const uint4*>(tK + off64(t, 32 * g4 + 8 * j));
          const uint32_t z4[4] = {zv.x, zv.y, zv.z, zv.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&z4[i]));
            zf[2 * i] = f.x;
            zf[2 * i + 1] = f.y;
          }
          ld8(wr + 8 * j, wf);
#pragma unroll
          for (int i = 0; i < 8; ++i) x[8 * j + i] *= rs * wf[i] * (zf[i] / (1.f + __expf(-zf[i])));
        }
      }
      if (live && ok) {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          reinterpret_cast<uint4*>(go)[4 * g4 + j] =
              make_uint4(pack_bf2(x[8 * j], x[8 * j + 1]), pack_bf2(x[8 * j + 2], x[8 * j + 3]),
                         pack_bf2(x[8 * j + 4], x[8 * j + 5]), pack_bf2(x[8 * j + 6], x[8 * j + 7]));
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (w == 0) tmem_dealloc(tmem, 256);
}

// ---- commit: S_m = e^{G_{m-1}} S0 + K~^T U over the first m = adv[b] rows ------------------------
struct CommitArgs {
  const bf16* kbuf; const bf16* ubuf; const float* gbuf;   // canvas outputs (rows b * n ..)
  float* ssm;
  const int* slot; const int* adv;
  int* err;
  int n, Hv;
};

__global__ void __launch_bounds__(NT) commit_kernel(const CommitArgs a) {
  __shared__ __align__(1024) uint8_t sk[T64];     // K~ [64 rows s][128 dk]
  __shared__ __align__(1024) uint8_t su[T64];     // U  [64 rows s][128 dv]
  __shared__ uint64_t bar;
  __shared__ uint32_t tslot;
  const int hv = blockIdx.x, b = blockIdx.y, t = threadIdx.x, w = t >> 5;
  const int m = min(max(a.adv[b], 0), a.n);
  if (t == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  if (w == 0) tmem_alloc(&tslot, 128);
  const float Gl = m > 0 ? a.gbuf[((int64_t)b * a.n + m - 1) * a.Hv + hv] : 0.f;
  // the state row of this thread (k index t) is loaded now, so its latency hides behind the rows
  // and the product; threads 0-63 stage row t of K~ and U with all their loads in flight
  float* S = a.ssm + (((int64_t)a.slot[b] * a.Hv + hv) * 128 + t) * 128;
  float4 s0[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) s0[j] = reinterpret_cast<const float4*>(S)[j];
  if (t < C) {
    if (t < m) {
      const int64_t row = (int64_t)b * a.n + t;
      uint4 xk[16], xu[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        xk[j] = reinterpret_cast<const uint4*>(a.kbuf + (row * a.Hv + hv) * 128)[j];
        xu[j] = reinterpret_cast<const uint4*>(a.ubuf + (row * a.Hv + hv) * 128)[j];
      }
      const float sc = __expf(Gl - a.gbuf[row * a.Hv + hv]);
      store_row(xk, sc, sk, t, nullptr);
      store_row(xu, 1.f, su, t, nullptr);
    } else {
      zero_row(sk, t, 128);
      zero_row(su, t, 128);
    }
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tslot;
  if (t == 0) {
    // M = dk (tile columns of K~, MN-major), N = dv, K = canvas rows
    mma(tmem, MN(smem_addr(sk), 0, H64), MN(smem_addr(su), 0, H64), 128, C, false);
    umma_commit(&bar);
  }
  const bool ok = mbar_wait(&bar, 0, a.err, 90);
  tc_fence_after();
  {  // every warp loads its 32 lanes (warp-collective tcgen05.ld); the state is written when ok
    const float gam = __expf(Gl);
#pragma unroll
    for (int g4 = 0; g4 < 4; ++g4) {
      float x[32];
      tld32(tmem + 32 * g4, x);
      if (!ok) continue;
      float4* p = reinterpret_cast<float4*>(S + 32 * g4);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float4 v = s0[8 * g4 + j];
        v.x = fmaf(gam, v.x, x[4 * j]);
        v.y = fmaf(gam, v.y, x[4 * j + 1]);
        v.z = fmaf(gam, v.z, x[4 * j + 2]);
        v.w = fmaf(gam, v.w, x[4 * j + 3]);
        p[j] = v;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (w == 0) tmem_dealloc(tmem, 128);
}

}  // namespace gdncv

int gdn_canvas_tc(const bf16* mixed, int64_t ldm, const bf16* ga, const bf16* gb, int64_t ldg, const float* A_log,
                  const float* dt_bias, const float* ssm, const int* slot, bf16* o, bf16* kbuf, bf16* ubuf, float* gbuf,
                  int B, int n, int n_clean, int Hk, int Hv, float scale, int* err, cudaStream_t st, const bf16* z,
                  int64_t ldz, const bf16* gnorm_w, float eps) {
  using namespace gdncv;
  if (n < 1 || n > C || Hv % Hk) return -1;
  CanvasArgs a{mixed, ldm, ga, gb, ldg, A_log, dt_bias, ssm, slot, o, z, ldz, gnorm_w, eps, kbuf, ubuf, gbuf, err,
               n, n_clean, Hk, Hv, scale};
  const int smem = CanvasSmem::TOTAL + 1024;
  static bool init = false;
  if (!init) {
    cudaFuncSetAttribute(canvas_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    init = true;
  }
  canvas_kernel<<<dim3(Hv, B), NT, smem, st>>>(a);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int gdn_commit_tc(const bf16* kbuf, const bf16* ubuf, const float* gbuf, float* ssm, const int* slot, const int* adv,
                  int B, int n, int Hv, int* err, cudaStream_t st) {
  using namespace gdncv;
  if (n < 1 || n > C) return -1;
  CommitArgs a{kbuf, ubuf, gbuf, ssm, slot, adv, err, n, Hv};
  commit_kernel<<<dim3(Hv, B), NT, 0, st>>>(a);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

}  // namespace trida
