// Shared pieces of the chunked gated-delta kernels (gdn_chunk.cu forward, gdn_chunk_bwd.cu
// backward): the tile algebra over swizzled 128 x 128 bf16 tiles, the per-row chunk metadata, the
// triangular inverse and the tensor-map helpers.  See gdn_chunk.cu for the design.
#pragma once

#include <cudaTypedefs.h>

#include "common.cuh"
#include "ops.h"
#include "sm100_common.cuh"

namespace trida {
namespace gdnc {

using namespace trida::sm100;

constexpr int D = 128;            // key / value head dim
constexpr int TR = 128;           // rows per tile
constexpr int NT = 128;           // threads (one per tile row / TMEM lane)
constexpr int TILE = 32768;       // bytes of a 128 x 128 bf16 tile
constexpr int SUB = 16384;        // one [128][64] swizzled half
constexpr int AF_BYTES = 128 * 64 * 4;   // fp32 A blocks: 128 rows x 64 chunk-local columns (one tile)

// Index of A-block element (row, chunk-local column): 64-float rows with the column XOR-ed by the
// row's low 5 bits, so a warp writing 32 rows of one column hits 32 banks while a warp reading one
// row (every thread the same element) is a broadcast.
__device__ __forceinline__ int af_idx(int row, int col) { return row * 64 + (col ^ (row & 31)); }

enum Mode { PREP = 0, NOISY = 1, OUT = 2 };

// ---- tile algebra --------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t toff(int r, int c) {
  return (uint32_t)(c >> 6) * SUB + sw128_offset(r, c & 63);
}

// K-major view: MN index = tile row (from row0), K index = tile column (from k0).  `half` is the
// byte distance between the two 64-column halves (SUB for a 128-row tile, rows * 128 otherwise).
__device__ __forceinline__ uint64_t kdesc(uint32_t base, int row0, int k0, uint32_t half) {
  return desc_sw128(base + (uint32_t)(k0 >> 6) * half + (uint32_t)row0 * 128u + (uint32_t)(k0 & 63) * 2u, 16, 1024);
}
// MN-major view: MN index = tile column, K index = tile row (from k0).
__device__ __forceinline__ uint64_t mdesc(uint32_t base, int k0, uint32_t half) {
  return desc_sw128(base + (uint32_t)k0 * 128u, half, 1024);
}

// D[128 x N] (+)= op(A) op(B) over K (multiple of 16).  a_mn / b_mn select the views above;
// a_row0 / b_row0 offset the MN rows of a K-major operand, a_k0 / b_k0 the K range.
struct Opnd {
  uint32_t base;
  int mn;      // 0: K-major view, 1: MN-major view
  int row0;    // K-major only: first MN row
  int k0;      // first K index
  uint32_t half;
};

__device__ __forceinline__ void mma(uint32_t d, Opnd a, Opnd b, int N, int K, bool acc) {
  const uint32_t id = idesc_bf16_f32(128, N, a.mn, b.mn);
  for (int kk = 0; kk < K / 16; ++kk) {
    const int ka = a.k0 + kk * 16, kb = b.k0 + kk * 16;
    const uint64_t ad = a.mn ? mdesc(a.base, ka, a.half) : kdesc(a.base, a.row0, ka, a.half);
    const uint64_t bd = b.mn ? mdesc(b.base, kb, b.half) : kdesc(b.base, b.row0, kb, b.half);
    umma_f16(d, ad, bd, id, (acc || kk > 0) ? 1u : 0u);
  }
}

__device__ __forceinline__ Opnd KM(uint32_t base, int row0 = 0, int k0 = 0, uint32_t half = SUB) {
  return Opnd{base, 0, row0, k0, half};
}
__device__ __forceinline__ Opnd MN(uint32_t base, int k0 = 0, uint32_t half = SUB) { return Opnd{base, 1, 0, k0, half}; }

// One row (128 fp32 TMEM columns from `col`) of an accumulator into registers.
__device__ __forceinline__ void ld_row128(uint32_t tmem, int col, float (&x)[128]) {
  const int w = threadIdx.x >> 5;
  const uint32_t a = tmem + ((uint32_t)(32 * w) << 16) + col;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t r[32];
    tmem_ld32(a + 32 * j, r);
    tmem_wait_ld();
#pragma unroll
    for (int i = 0; i < 32; ++i) x[32 * j + i] = __uint_as_float(r[i]);
  }
}

__device__ __forceinline__ uint32_t pack_bf2(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Row r of a tile from 128 fp32 values (first n columns; the rest written as zero).
__device__ __forceinline__ void st_row(uint8_t* tile, int r, const float (&x)[128]) {
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    uint4 v;
    v.x = pack_bf2(x[8 * j + 0], x[8 * j + 1]);
    v.y = pack_bf2(x[8 * j + 2], x[8 * j + 3]);
    v.z = pack_bf2(x[8 * j + 4], x[8 * j + 5]);
    v.w = pack_bf2(x[8 * j + 6], x[8 * j + 7]);
    *reinterpret_cast<uint4*>(tile + toff(r, 8 * j)) = v;
  }
}

__device__ __forceinline__ void ld_row_bf(const uint8_t* tile, int r, float (&x)[128]) {
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const uint4 v = *reinterpret_cast<const uint4*>(tile + toff(r, 8 * j));
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&w[i]);
      const float2 f = __bfloat1622float2(h);
      x[8 * j + 2 * i] = f.x;
      x[8 * j + 2 * i + 1] = f.y;
    }
  }
}

__device__ __forceinline__ void st_col(uint8_t* tile, int c, const float (&x)[128]) {
#pragma unroll
  for (int r = 0; r < 128; ++r) *reinterpret_cast<bf16*>(tile + toff(r, c)) = __float2bfloat16(x[r]);
}

__device__ __forceinline__ float ld_el(const uint8_t* tile, int r, int c) {
  return __bfloat162float(*reinterpret_cast<const bf16*>(tile + toff(r, c)));
}

// ---- 32-column groups -----------------------------------------------------------------------------
// Row passes walk a 128-column row in groups of 32 columns with a rolled outer loop: the unrolled
// inner body stays small (instruction cache) and 32 values live in registers instead of 128.
__device__ __forceinline__ uint32_t lane_base() { return (uint32_t)(32 * (threadIdx.x >> 5)) << 16; }

__device__ __forceinline__ void tm_ld32(uint32_t acc, int g, float (&x)[32]) {
  uint32_t v[32];
  tmem_ld32(acc + lane_base() + 32 * g, v);
  tmem_wait_ld();
#pragma unroll
  for (int i = 0; i < 32; ++i) x[i] = __uint_as_float(v[i]);
}

__device__ __forceinline__ void tm_st32(uint32_t acc, int g, const float (&x)[32]) {
  uint32_t v[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(x[i]);
  tmem_st32(acc + lane_base() + 32 * g, v);
}

__device__ __forceinline__ void sm_st32(uint8_t* tile, int r, int g, const float (&x)[32], float sc = 1.f) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint4 v;
    v.x = pack_bf2(x[8 * j] * sc, x[8 * j + 1] * sc);
    v.y = pack_bf2(x[8 * j + 2] * sc, x[8 * j + 3] * sc);
    v.z = pack_bf2(x[8 * j + 4] * sc, x[8 * j + 5] * sc);
    v.w = pack_bf2(x[8 * j + 6] * sc, x[8 * j + 7] * sc);
    *reinterpret_cast<uint4*>(tile + toff(r, 32 * g + 8 * j)) = v;
  }
}

__device__ __forceinline__ void sm_zero32(uint8_t* tile, int r, int g) {
  const uint4 z = make_uint4(0, 0, 0, 0);
#pragma unroll
  for (int j = 0; j < 4; ++j) *reinterpret_cast<uint4*>(tile + toff(r, 32 * g + 8 * j)) = z;
}

__device__ __forceinline__ void sm_ld32(const uint8_t* tile, int r, int g, float (&x)[32]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint4 v = *reinterpret_cast<const uint4*>(tile + toff(r, 32 * g + 8 * j));
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
      x[8 * j + 2 * i] = f.x;
      x[8 * j + 2 * i + 1] = f.y;
    }
  }
}

__device__ __forceinline__ void gm_st32(bf16* dst, const float (&x)[32], float sc = 1.f) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint4 v;
    v.x = pack_bf2(x[8 * j] * sc, x[8 * j + 1] * sc);
    v.y = pack_bf2(x[8 * j + 2] * sc, x[8 * j + 3] * sc);
    v.z = pack_bf2(x[8 * j + 4] * sc, x[8 * j + 5] * sc);
    v.w = pack_bf2(x[8 * j + 6] * sc, x[8 * j + 7] * sc);
    reinterpret_cast<uint4*>(dst)[j] = v;
  }
}

// Transposed group store: rows 32g..32g+31 of tile column c.
__device__ __forceinline__ void sm_st_col32(uint8_t* tile, int c, int g, const float (&x)[32]) {
#pragma unroll
  for (int i = 0; i < 32; ++i) *reinterpret_cast<bf16*>(tile + toff(32 * g + i, c)) = __float2bfloat16(x[i]);
}

// Sum of x[i] over the warp's 32 lanes for every i; lane l returns the sum for i = l (31 shuffles).
__device__ __forceinline__ float warp_colsum32(float (&x)[32]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int m = 16, n = 16; m >= 1; m >>= 1, n >>= 1) {
    const bool hi = (lane & m) != 0;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      if (i < n) {
        const float send = hi ? x[i] : x[n + i];
        const float keep = hi ? x[n + i] : x[i];
        x[i] = keep + __shfl_xor_sync(0xffffffffu, send, m);
      }
    }
  }
  return x[0];
}

// Chunk-local C x C matrices are block diagonal in a 128-row tile: a row's nonzero columns lie in
// its window of W = max(C, 32) columns (warp-uniform), i.e. groups [win_g0, win_g0 + W / 32).
template <int C>
struct Win {
  static constexpr int W = C < 32 ? 32 : C;
  static constexpr int NG = W / 32;
  __device__ static int g0() { return ((int)threadIdx.x / W) * NG; }
};

// ---- arguments ------------------------------------------------------------------------------------
struct Args {
  int B, T, Hk, Hv;
  int mode;                 // layout: 0 causal, 1 two-stream
  int L, V;                 // two-stream geometry (stream length, noisy views)
  int nch;                  // clean chunks per row
  int tok_clean, tok_noisy; // token-causal read-out of the clean / noisy streams
  const uint8_t* doc;       // [B, Lc] document starts of the clean stream (or null)
  const float* gb;          // [B*T, Hv, 2]: log-decay g, beta
  bf16* o;                  // [B*T, Hv*D]
  bf16* ckpt;               // [B, Hv, nch, D, D] clean chunk-start states (k rows, v columns)
  float* gamma;             // [B, Hv, nch] chunk decay carry_last * e^{G_last}
  float* final_state;       // optional [B, Hv, D, D] fp32 state after the last clean token
  bf16* wn;                 // [B*T, Hv, D] -W rows (clean stream)
  bf16* ut;                 // [B*T, Hv, D] U~ rows
  bf16* kt;                 // [B*T, Hv, D] K~ rows
  bf16* u;                  // [B*T, Hv, D] U rows (clean rows by the scan, noisy rows by the noisy kernel)
  int* err;
  // backward
  const bf16* o_fwd;        // [B*T, Hv*D] forward output (dG of the read-out decay: dO . O)
  const bf16* d_o;          // [B*T, Hv*D]
  bf16* du0;                // [B*T, Hv, D] P^T dO of clean rows (scan input)
  bf16* du;                 // [B*T, Hv, D] dU (clean rows by the scan, noisy rows by bwd0)
  bf16* qg;                 // [B*T, Hv, D] carry e^{Gr} q rows of the clean stream
  bf16* ds0;                // [B, Hv, nch, D, D] noisy gradient w.r.t. each clean chunk-start state
  bf16* dckpt;              // [B, Hv, nch, D, D] gradient w.r.t. each clean chunk's end state
  bf16* dpe; bf16* dae; bf16* dw; bf16* tt;   // [B*T, Hv, D] bwd1 -> bwd2 rows
  float* sc;                // [B*T, Hv, 2] bwd1 partial d beta, d G
  float* dpart;             // [B*T, Hv, RED]: dq | dk | dbeta | dg (per value head)
  bf16* dv; int64_t lddv;   // value-gradient rows (head columns at hv * D)
  const bf16* mixed; int64_t ldm;   // conv output (v rows for d beta)
  const bf16* qk_rows;              // [B*T, Hk, 2, D] normalised q (times scale) / k
};

__device__ __forceinline__ int clean_len(const Args& a) { return a.mode ? a.L : a.T; }

// Per-tile stream geometry.
struct TileGeo {
  int b, hv, hk;
  int stream;               // 0 clean / causal, 1.. noisy view
  int p0;                   // first stream position of the tile
  int Ls;                   // stream length
  int t0;                   // first row of the tile inside batch row b
  bool tok;                 // token-causal read-out
};

__device__ __forceinline__ void store_row_bf(bf16* dst, const float (&x)[128], float scale) {
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    uint4 v;
    v.x = pack_bf2(x[8 * j] * scale, x[8 * j + 1] * scale);
    v.y = pack_bf2(x[8 * j + 2] * scale, x[8 * j + 3] * scale);
    v.z = pack_bf2(x[8 * j + 4] * scale, x[8 * j + 5] * scale);
    v.w = pack_bf2(x[8 * j + 6] * scale, x[8 * j + 7] * scale);
    reinterpret_cast<uint4*>(dst)[j] = v;
  }
}

// ---- per-row metadata ------------------------------------------------------------------------------
struct Meta {
  float* g; float* beta; float* G; float* Gr; float* carry; float* kts; int* seg; int* rd; int* rs; float* gam;
  static constexpr int BYTES = 10 * 128 * 4;
};

__device__ __forceinline__ Meta carve_meta(uint8_t* p) {
  Meta m;
  float* f = reinterpret_cast<float*>(p);
  m.g = f; m.beta = f + 128; m.G = f + 256; m.Gr = f + 384; m.carry = f + 512; m.kts = f + 640;
  m.seg = reinterpret_cast<int*>(f + 768); m.rd = reinterpret_cast<int*>(f + 896);
  m.rs = reinterpret_cast<int*>(f + 1024); m.gam = f + 1152;
  return m;
}

// Thread r fills the metadata of tile row r: decay / beta (0 past the stream end), segment starts
// from document starts, the segmented cumulative log-decay G, read-out row rd, Gr = G[rd], carry,
// the K~ row scale and (thread of each chunk's first row) the chunk decay.
template <int C>
__device__ void tile_meta(const Args& a, const TileGeo& t, const Meta& m) {
  const int r = threadIdx.x;
  const int p = t.p0 + r;
  float g = 0.f, be = 0.f;
  int rs = 0;
  if (p < t.Ls) {
    const int64_t row = (int64_t)t.b * a.T + t.t0 + r;
    const float2 v = *reinterpret_cast<const float2*>(a.gb + (row * a.Hv + t.hv) * 2);
    g = v.x;
    be = v.y;
    if (a.doc != nullptr) {
      const bool start = a.doc[(int64_t)t.b * clean_len(a) + p] != 0;   // noisy views share positions
      rs = (t.stream == 0 || (r % C) == 0) ? (int)start : 0;
    }
  }
  m.g[r] = g;
  m.beta[r] = be;
  m.rs[r] = rs;
  __syncthreads();
  const int cs = (r / C) * C;
  int seg = 0, sst = cs;
  for (int j = cs + 1; j <= r; ++j)
    if (m.rs[j]) { ++seg; sst = j; }
  float G = 0.f;
  for (int j = sst; j <= r; ++j) G += m.g[j];
  int rd = r;
  if (!t.tok) {
    rd = cs + C - 1;
    for (int j = r + 1; j < cs + C; ++j)
      if (m.rs[j]) { rd = j - 1; break; }
  }
  m.G[r] = G;
  m.seg[r] = seg;
  m.rd[r] = rd;
  m.carry[r] = (seg == 0 && !m.rs[cs]) ? 1.f : 0.f;
  __syncthreads();
  const int last = cs + C - 1;
  m.Gr[r] = m.G[rd];
  m.kts[r] = (m.seg[r] == m.seg[last]) ? __expf(m.G[last] - G) : 0.f;
  if (r == cs) m.gam[r / C] = m.carry[last] * __expf(m.G[last]);
  __syncthreads();
}

// Column j of T = (I + A)^-1 for the chunk holding tile column j (forward substitution over the
// fp32 A blocks, chunk-local columns, see af_idx), written into the T tile as bf16 (zero outside
// the chunk's diagonal block).
template <int C>
__device__ __forceinline__ void invert_column(const float* Af, uint8_t* Tt) {
  const int j = threadIdx.x, cs = (j / C) * C, jl = j - cs;
  float x[C];
#pragma unroll
  for (int t = 0; t < C; ++t) x[t] = (t == jl) ? 1.f : 0.f;
#pragma unroll
  for (int t = 1; t < C; ++t) {
    const int row = cs + t;
    float s = 0.f;
#pragma unroll
    for (int u = 0; u < t; ++u) s = fmaf(Af[af_idx(row, u)], x[u], s);
    if (t > jl) x[t] = -s;
  }
#pragma unroll
  for (int t = 0; t < C; ++t) *reinterpret_cast<bf16*>(Tt + toff(cs + t, j)) = __float2bfloat16(x[t]);
  const bf16 z = __float2bfloat16(0.f);
  for (int r = 0; r < 128; ++r)
    if (r < cs || r >= cs + C) *reinterpret_cast<bf16*>(Tt + toff(r, j)) = z;
}

// ---- host -----------------------------------------------------------------------------------------
inline PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  inline PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

inline bool encode(CUtensorMap* m, const void* base, const cuuint64_t (&dims)[4], const cuuint64_t (&strides)[3],
                   int box1, int box2) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint32_t box[4] = {64, (cuuint32_t)box1, (cuuint32_t)box2, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  cuuint64_t d[4] = {dims[0], dims[1], dims[2], dims[3]};
  cuuint64_t st[3] = {strides[0], strides[1], strides[2]};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), d, st, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// bf16 [B][T][H][D]: coordinates (d, h, t, b); box 64 x 1 head x box_rows tokens.  Tokens past T
// read as zero.
inline bool map_heads(CUtensorMap* m, const void* base, int B, int T, int H, int box_rows) {
  const cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)T, (cuuint64_t)B};
  const cuuint64_t strides[3] = {(cuuint64_t)D * 2, (cuuint64_t)H * D * 2, (cuuint64_t)T * H * D * 2};
  return encode(m, base, dims, strides, 1, box_rows);
}

// bf16 [B][T][ld] (first `cols` columns): coordinates (col, t, b, 0); box 64 x box_rows tokens.
inline bool map_cols(CUtensorMap* m, const void* base, int B, int T, int64_t cols, int64_t ld, int box_rows) {
  const cuuint64_t dims[4] = {(cuuint64_t)cols, (cuuint64_t)T, (cuuint64_t)B, 1};
  const cuuint64_t strides[3] = {(cuuint64_t)ld * 2, (cuuint64_t)T * ld * 2, (cuuint64_t)B * T * ld * 2};
  return encode(m, base, dims, strides, box_rows, 1);
}


}  // namespace gdnc
}  // namespace trida
