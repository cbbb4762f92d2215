// Persistent bf16 tensor-core GEMM for sm_100a written directly against tcgen05 / TMA.
//
//   D[M,N] = alpha * op(A) op(B) + beta * C        (fp32 accumulation in TMEM, D bf16 or fp32)
//
// One CTA per SM walks output tiles of 128 x 256 (grouped raster for L2 reuse).  Warp roles:
//   warp 0      TMA producer: 64-deep K slices of A and B into a 4-stage shared-memory ring
//               (plain per-CTA tensor loads: every CTA fetches its own tiles);
//   warp 1      MMA issuer (one thread): 4 x tcgen05.mma (K = 16) per K slice into one of two
//               TMEM accumulators (128 lanes x 256 fp32 columns each), so the epilogue of tile i
//               overlaps the mainloop of tile i + 1;
//   warps 2-5   epilogue: tcgen05.ld 32 columns at a time, alpha / beta * C, convert, store.
// Fused all-reduce epilogue (tensor-parallel row-parallel layers, ``gemm_bf16_allreduce``): the
// epilogue warps push each tile's bf16 partial from registers into every rank's receive buffer over
// NVLink (plain stores to peer memory), release the TMEM accumulator to the next tile, bump one
// arrival counter per (tile, warp) on every rank, then wait until all ranks' partials of their rows
// have arrived in this GPU's own buffer, sum them (+ residual) and TMA-store the result: the
// GEMM and its all-reduce are one kernel, and the exchange of tile i overlaps the mainloop of
// tile i + 1.  Receive buffers and counters alternate between two parities by a device-side call
// counter (graph-capturable); a waiter resets its counter after use, which is safe because a rank
// can only start the next same-parity call after this rank has finished the current one.
// Operand majorness follows the caller's row-major tensors: K-major operands are loaded with a
// 64-element K box (UMMA K-major SWIZZLE_128B), MN-major operands with a 64-element MN box
// (UMMA MN-major SWIZZLE_128B; LBO = one 64-wide MN atom).  Every mbarrier wait is bounded.
#include <cudaTypedefs.h>

#include "common.cuh"
#include "gemm_sm100.cuh"
#include "sm100_common.cuh"

namespace trida {
namespace gemm100 {

using namespace sm100;

constexpr int BN = 256, BK = 64;
constexpr int NTHREADS = 192;
constexpr int B_BYTES = BN * BK * 2;     // 32 KB
constexpr int GROUP_M = 16;

// MH = 128-row halves per tile: MH = 1 -> 128 x 256 tiles, 4-stage ring, two TMEM accumulators
// (the epilogue of one tile overlaps the mainloop of the next); MH = 2 -> 256 x 256 tiles (two
// MMAs share every B slice, 1.5x the FLOPs per byte staged), 3-stage ring, one accumulator
// spanning all 512 TMEM columns.
template <int MH>
struct Cfg {
  static constexpr int BM = 128 * MH;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = MH == 1 ? 4 : 3;
  static constexpr int NACC = MH == 1 ? 2 : 1;
  // epilogue staging: 4 warps x 2 buffers x (32 rows x 128 B), TMA-stored (128B swizzle)
  static constexpr int EPI_BYTES = 4 * 2 * 4096;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + EPI_BYTES + 256 + 1024;
};

struct Params {
  int M, N, K;
  int a_kmajor, b_kmajor;
  void* D;
  int64_t ldd;
  const void* C;
  int64_t ldc;
  float alpha, beta;
  int d_fp32;
  int* err;
  int splits, kb_per;     // split-K: units = tiles * splits, each over kb_per K blocks
  float* ws;              // split-K partials [splits, M, N] fp32 (splits > 1)
  // fused all-reduce (ar_world > 1): per destination rank, its receive buffer
  // [2 parities][world][mcap][N] bf16 and its arrival counters [2][tiles_cap][4 warps]
  int ar_world, ar_rank, ar_tiles_cap;
  int64_t ar_mcap;
  bf16* ar_recv[8];
  unsigned* ar_flag[8];
  unsigned* ar_ctr;       // this rank's call counter (the call's epoch = *ar_ctr + 1)
  unsigned* ar_done;      // CTAs finished in this call (the last one advances ar_ctr)
  float* ar_ws;           // split-K: fp32 partial tiles [tiles * splits][128][256] (this GPU)
  unsigned* ar_tile_ctr;  // split-K: arrivals per (tile, epilogue warp), reset by the last arrival
  // SwiGLU mode (glu_f > 0, TN, B = [gate; up] with glu_f rows each): a tile covers 128 features,
  // its B slice stacks the 128 gate rows over the matching 128 up rows, and the epilogue writes
  // both halves back to D = gu [M, 2 glu_f] plus E = silu(gate) * up [M, glu_f]
  int glu_f;
  // argmax mode (am_val != null): D is not written; each output tile leaves, per row, the max of its
  // columns and that column's index in am_val / am_idx [M, am_ld] (column = N tile); a second
  // kernel reduces the row's tiles (greedy tokens without materialising the logits)
  float* am_val;
  int* am_idx;
  int am_ld;
};

__device__ __forceinline__ void red_release_sys(unsigned* p, unsigned v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Poll a counter until it reaches `target`; gives up after kWaitLimitNs (error word set).
__device__ __forceinline__ bool wait_count(const unsigned* f, unsigned target, int* err, int code) {
  const uint64_t t0 = global_ns();
  for (uint32_t it = 0;; ++it) {
    if (ld_acquire_sys(f) >= target) return true;
    if ((it & 255u) == 255u) {
      if (global_ns() - t0 > kWaitLimitNs) {
        atomicExch(err, code);
        return false;
      }
      __nanosleep(200);
    }
  }
}

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n" ::
          "r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];\n" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_addr(src)), "r"(c0), "r"(c1)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;\n" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;\n" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory"); }

__device__ __forceinline__ void tile_coords(int tile, int mt, int nt, int bm, int& m0, int& n0) {
  const int per_group = GROUP_M * nt;
  const int g = tile / per_group;
  const int first_m = g * GROUP_M;
  const int gm = (mt - first_m) < GROUP_M ? (mt - first_m) : GROUP_M;
  const int in = tile % per_group;
  m0 = (first_m + in % gm) * bm;
  n0 = (in / gm) * BN;
}

// Load one K slice of an operand tile.  K-major: rows x 64 K  (box {64, rows}, rows <= 256).
// MN-major: 64 K rows x MN (box {64 MN, 64 K}); `width` MN elements in 64-wide atoms.
__device__ __forceinline__ void load_operand(unsigned char* dst, const CUtensorMap* map, uint64_t* bar, int kmajor,
                                             int mn0, int k0, int width) {
  if (kmajor) {
    tma_load_2d(dst, map, bar, k0, mn0);
  } else {
    for (int j = 0; j < width / 64; ++j) tma_load_2d(dst + j * (BK * 128), map, bar, mn0 + j * 64, k0);
  }
}

__device__ __forceinline__ uint64_t operand_desc(uint32_t base, int kmajor, int kk) {
  // kk = 16-element K step inside the 64-wide slice
  if (kmajor) return desc_sw128(base + kk * 32, 16, 1024);
  return desc_sw128(base + kk * 2048, BK * 128, 1024);
}

template <int MH>
__global__ void __launch_bounds__(NTHREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmD, const __grid_constant__ CUtensorMap tmC,
                const __grid_constant__ CUtensorMap tmE, const Params p) {
  using C_ = Cfg<MH>;
  constexpr int BM = C_::BM, STAGES = C_::STAGES, NACC = C_::NACC;
  constexpr int A_BYTES = C_::A_BYTES, STAGE_BYTES = C_::STAGE_BYTES;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  unsigned char* epi = smem + STAGES * STAGE_BYTES;                 // 1024-aligned staging
  uint64_t* bars = reinterpret_cast<uint64_t*>(epi + C_::EPI_BYTES);
  uint64_t* full = bars;                       // [STAGES]
  uint64_t* empty = bars + STAGES;             // [STAGES]
  uint64_t* acc_full = bars + 2 * STAGES;      // [NACC]
  uint64_t* acc_empty = bars + 2 * STAGES + 2; // [NACC]
  uint64_t* drain = bars + 2 * STAGES + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 6);
  uint64_t* cbar = bars + 2 * STAGES + 8;      // [4 warps x 2 buffers] C-tile loads

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mt = (p.M + BM - 1) / BM, nt = p.glu_f > 0 ? (p.glu_f + 127) / 128 : (p.N + BN - 1) / BN;
  const int units = mt * nt * p.splits;
  const int kb = (p.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < NACC; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    mbar_init(drain, 1);
    for (int i = 0; i < 8; ++i) mbar_init(&cbar[i], 1);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tmA);
      prefetch_tmap(&tmB);
      int it = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < units; u += gridDim.x) {
        int m0, n0;
        tile_coords(u / p.splits, mt, nt, BM, m0, n0);
        const int kbeg = (u % p.splits) * p.kb_per, kend = min(kb, kbeg + p.kb_per);
        for (int k = kbeg; k < kend; ++k, ++it) {
          const int s = it % STAGES;
          if (it >= STAGES && !(ok = mbar_wait(&empty[s], ((it / STAGES) - 1) & 1, p.err, 101))) break;
          unsigned char* st = smem + s * STAGE_BYTES;
          mbar_expect_tx(&full[s], STAGE_BYTES);
          load_operand(st, &tmA, &full[s], p.a_kmajor, m0, k * BK, BM);
          if (p.glu_f > 0) {   // 128 gate rows, then the 128 up rows of the same features
            tma_load_2d(st + A_BYTES, &tmB, &full[s], k * BK, n0 >> 1);
            tma_load_2d(st + A_BYTES + 128 * 128, &tmB, &full[s], k * BK, p.glu_f + (n0 >> 1));
          } else {
            load_operand(st + A_BYTES, &tmB, &full[s], p.b_kmajor, n0, k * BK, BN);
          }
        }
      }
      // the final (up to STAGES) loads must land before the CTA retires
      for (int j = (it > STAGES ? it - STAGES : 0); ok && j < it; ++j)
        mbar_wait(&full[j % STAGES], (j / STAGES) & 1, p.err, 102);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(128, BN, p.a_kmajor ? 0 : 1, p.b_kmajor ? 0 : 1);
      int it = 0, t = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < units; u += gridDim.x, ++t) {
        const int ab = t % NACC;
        if (t >= NACC && !(ok = mbar_wait(&acc_empty[ab], ((t / NACC) - 1) & 1, p.err, 103))) break;
        tc_fence_after();
        const uint32_t dcol = tmem + ab * BN;
        const int kbeg = (u % p.splits) * p.kb_per, kend = min(kb, kbeg + p.kb_per);
        for (int k = kbeg; k < kend; ++k, ++it) {
          const int s = it % STAGES;
          if (!(ok = mbar_wait(&full[s], (it / STAGES) & 1, p.err, 104))) break;
          tc_fence_after();
          const uint32_t a_base = smem_addr(smem + s * STAGE_BYTES);
          const uint32_t b_base = a_base + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t bdesc = operand_desc(b_base, p.b_kmajor, kk);
#pragma unroll
            for (int h = 0; h < MH; ++h)   // rows h*128.. of the A tile start 16 KB further in
              umma_f16(dcol + h * BN, operand_desc(a_base + h * 16384, p.a_kmajor, kk), bdesc, idesc,
                       (k > kbeg || kk > 0) ? 1u : 0u);
          }
          umma_commit(&empty[s]);
        }
        if (ok) umma_commit(&acc_full[ab]);
      }
      umma_commit(drain);
      mbar_wait(drain, 0, p.err, 105);
    }
  } else {
    // epilogue warps 2..5: TMEM lane quarter = warp % 4
    const int q = warp & 3;
    const int r = q * 32 + lane;                       // accumulator row (TMEM lane)
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    int ebuf = 0;
    uint32_t cpar[2] = {0u, 0u};
    int t = 0;
    const bool fused = p.ar_world > 1;
    const unsigned epoch = fused ? *reinterpret_cast<volatile unsigned*>(p.ar_ctr) + 1u : 0u;
    const int par = (int)(epoch & 1u);
    for (int u = blockIdx.x; u < units; u += gridDim.x, ++t) {
      const int ab = t % NACC;
      if (!mbar_wait(&acc_full[ab], (t / NACC) & 1, p.err, 106)) break;
      tc_fence_after();
      int m0, n0;
      tile_coords(u / p.splits, mt, nt, BM, m0, n0);
      if (fused) {
        const int W = p.ar_world;
        const int tile = u / p.splits;
        const bool ksplit = p.splits > 1;                // MH == 1 whenever the all-reduce is fused
        if (ksplit) {
          // ---- phase 0 (split K): stash this split's fp32 rows; the warp arriving last for these
          // 32 rows of the tile sums all splits and carries on, the others are done with the tile
          float* wrow = p.ar_ws + ((int64_t)u * 128 + r) * BN;     // u = tile * splits + split
#pragma unroll 1
          for (int c = 0; c < BN / 32; ++c) {
            uint32_t v[32];
            tmem_ld32(tmem + ab * BN + lane_off + c * 32, v);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 32; j += 4)
              *reinterpret_cast<float4*>(wrow + c * 32 + j) =
                  make_float4(__uint_as_float(v[j]), __uint_as_float(v[j + 1]), __uint_as_float(v[j + 2]),
                              __uint_as_float(v[j + 3]));
          }
          tc_fence_before();
          mbar_arrive(&acc_empty[ab]);
          __threadfence();
          __syncwarp();
          int last = 0;
          if (lane == 0) last = atomicAdd(p.ar_tile_ctr + tile * 4 + q, 1u) == (unsigned)(p.splits - 1);
          last = __shfl_sync(0xffffffffu, last, 0);
          if (!last) continue;
          __threadfence();
          if (lane == 0) p.ar_tile_ctr[tile * 4 + q] = 0u;
        }
        // ---- phase 1: this rank's partial rows -> every rank's receive buffer (slot ar_rank).
        // Each 32-row x 64-column chunk is packed to bf16 in the warp's swizzled staging tile, then
        // copied out by 8 lanes per row so every store instruction writes four whole 128-byte row
        // segments (NVLink-friendly) instead of 32 scattered 16-byte pieces.
        const int row0 = m0 + q * 32;                    // MH == 1 whenever the all-reduce is fused
        if (lane == 0) bulk_wait_read0();                // no earlier TMA store still reads staging
        __syncwarp();
#pragma unroll 1
        for (int ch = 0; ch < BN / 64; ++ch) {
          float f[64];
          if (ksplit) {
#pragma unroll
            for (int j = 0; j < 64; ++j) f[j] = 0.f;
            for (int sidx = 0; sidx < p.splits; ++sidx) {
              const float4* src = reinterpret_cast<const float4*>(
                  p.ar_ws + ((int64_t)(tile * p.splits + sidx) * 128 + r) * BN + ch * 64);
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const float4 x = src[j];
                f[4 * j] += x.x; f[4 * j + 1] += x.y; f[4 * j + 2] += x.z; f[4 * j + 3] += x.w;
              }
            }
          } else {
            uint32_t v0[32], v1[32];
            tmem_ld32(tmem + ab * BN + lane_off + ch * 64, v0);
            tmem_ld32(tmem + ab * BN + lane_off + ch * 64 + 32, v1);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 32; ++j) { f[j] = __uint_as_float(v0[j]); f[32 + j] = __uint_as_float(v1[j]); }
          }
          const int col0 = n0 + ch * 64;
          if (row0 >= p.M || col0 >= p.N) continue;      // warp-uniform
          unsigned char* sb = epi + q * 8192 + (ch & 1) * 4096;
          unsigned char* rowp = sb + lane * 128;
#pragma unroll
          for (int j = 0; j < 8; ++j)
            *reinterpret_cast<uint4*>(rowp + ((j ^ (lane & 7)) << 4)) =
                make_uint4(pack_bf16x2(f[8 * j], f[8 * j + 1]), pack_bf16x2(f[8 * j + 2], f[8 * j + 3]),
                           pack_bf16x2(f[8 * j + 4], f[8 * j + 5]), pack_bf16x2(f[8 * j + 6], f[8 * j + 7]));
          __syncwarp();
          const int seg = lane & 7;
#pragma unroll 1
          for (int it = 0; it < 8; ++it) {
            const int rr = it * 4 + (lane >> 3);
            if (row0 + rr >= p.M) continue;
            const uint4 val = *reinterpret_cast<const uint4*>(sb + rr * 128 + ((seg ^ (rr & 7)) << 4));
            const int64_t off = ((int64_t)(par * W + p.ar_rank) * p.ar_mcap + row0 + rr) * p.N + col0 + seg * 8;
#pragma unroll 1
            for (int d = 0; d < W; ++d)
              *reinterpret_cast<uint4*>(p.ar_recv[(p.ar_rank + d) % W] + off) = val;
          }
          __syncwarp();
        }
        if (!ksplit) {
          tc_fence_before();
          mbar_arrive(&acc_empty[ab]);               // the accumulator is free for the next tile
        }
        const int64_t fidx = ((int64_t)par * p.ar_tiles_cap + tile) * 4 + q;
        asm volatile("fence.acq_rel.sys;\n" ::: "memory");
        __syncwarp();
        if (lane == 0)
          for (int d = 0; d < W; ++d) red_release_sys(p.ar_flag[(p.ar_rank + d) % W] + fidx, 1u);
        // ---- phase 2: wait for every rank's partial of this warp's rows, sum (+ C), TMA-store D
        int ok = 1;
        if (lane == 0) {
          unsigned* fl = p.ar_flag[p.ar_rank] + fidx;
          ok = wait_count(fl, (unsigned)W, p.err, 110) ? 1 : 0;
          if (ok) *reinterpret_cast<volatile unsigned*>(fl) = 0u;
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        __syncwarp();
        if (!ok) continue;
        const bool use_c = p.C != nullptr && p.beta != 0.f;
        const bf16* own = p.ar_recv[p.ar_rank];
        ebuf = 0;
#pragma unroll 1
        for (int ch = 0; ch < BN / 64; ++ch) {
          const int col0 = n0 + ch * 64;
          if (row0 >= p.M || col0 >= p.N) continue;      // warp-uniform
          unsigned char* sb = epi + q * 8192 + ebuf * 4096;
          if (lane == 0) bulk_wait_read1();
          __syncwarp();
          if (use_c) {
            if (lane == 0) {
              mbar_expect_tx(&cbar[q * 2 + ebuf], 4096);
              tma_load_2d(sb, &tmC, &cbar[q * 2 + ebuf], col0, row0);
            }
            mbar_wait(&cbar[q * 2 + ebuf], cpar[ebuf], p.err, 107);
            cpar[ebuf] ^= 1;
          }
          const int seg = lane & 7;
#pragma unroll 1
          for (int it = 0; it < 8; ++it) {               // 8 lanes per row: coalesced 128-byte reads
            const int rr = it * 4 + (lane >> 3);
            float o[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            if (row0 + rr < p.M) {
#pragma unroll 1
              for (int sidx = 0; sidx < W; ++sidx) {
                float x[8];
                load8(own + ((int64_t)(par * W + sidx) * p.ar_mcap + row0 + rr) * p.N + col0 + seg * 8, x);
#pragma unroll
                for (int e = 0; e < 8; ++e) o[e] += x[e];
              }
            }
            bf16* cp = reinterpret_cast<bf16*>(sb + rr * 128 + ((seg ^ (rr & 7)) << 4));
#pragma unroll
            for (int e = 0; e < 8; ++e) o[e] *= p.alpha;
            if (use_c) {
              float cv[8];
              load8(cp, cv);
#pragma unroll
              for (int e = 0; e < 8; ++e) o[e] += p.beta * cv[e];
            }
            store8(cp, o);
          }
          fence_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmD, sb, col0, row0);
            bulk_commit();
          }
          ebuf ^= 1;
        }
        continue;
      }
#pragma unroll 1
      for (int h = 0; h < MH; ++h) {
      const uint32_t acc = tmem + (ab + h) * BN + lane_off;
      const int row = m0 + h * 128 + r;
      const bool rok = row < p.M;
      if (p.am_val != nullptr) {
        // argmax tile: the row's best column among this tile's (first index on ties)
        float best = -INFINITY;
        int bidx = n0;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t v[32];
          tmem_ld32(acc + c * 32, v);
          tmem_wait_ld();
          const int col0 = n0 + c * 32;
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float x = __uint_as_float(v[j]);
            if (col0 + j < p.N && x > best) {
              best = x;
              bidx = col0 + j;
            }
          }
        }
        if (rok) {
          p.am_val[(int64_t)row * p.am_ld + n0 / BN] = best;
          p.am_idx[(int64_t)row * p.am_ld + n0 / BN] = bidx;
        }
        continue;
      }
      if (p.splits > 1) {
        // split-K partial: raw fp32 accumulator to the workspace (alpha / beta applied by the reduce)
        float* wrow = p.ws + ((int64_t)(u % p.splits) * p.M + row) * p.N;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t v[32];
          tmem_ld32(acc + c * 32, v);
          tmem_wait_ld();
          const int col0 = n0 + c * 32;
          if (!rok || col0 >= p.N) continue;
          if (col0 + 32 <= p.N && (p.N & 3) == 0) {
#pragma unroll
            for (int j = 0; j < 32; j += 4)
              *reinterpret_cast<float4*>(wrow + col0 + j) =
                  make_float4(__uint_as_float(v[j]), __uint_as_float(v[j + 1]), __uint_as_float(v[j + 2]),
                              __uint_as_float(v[j + 3]));
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (col0 + j < p.N) wrow[col0 + j] = __uint_as_float(v[j]);
          }
        }
        continue;
      }
      if (p.glu_f > 0) {
        // SwiGLU tile: accumulator columns [0, 128) are the gate features nf0.., [128, 256) the up
        // features of the same indices.  Each 64-column chunk is packed to bf16 and TMA-stored at
        // its natural column of gu; a gate chunk stays in registers until its up chunk is read and
        // gives silu(gate) * up from the bf16-rounded values, TMA-stored into E.
        const int row0 = m0 + h * 128 + q * 32;
        const int nf0 = n0 >> 1;
        auto stage_store = [&](const uint32_t (&w)[32], const CUtensorMap* map, int col) {
          unsigned char* sb = epi + q * 8192 + ebuf * 4096;
          if (lane == 0) bulk_wait_read1();           // the store issued from sb two chunks ago has read it
          __syncwarp();
          unsigned char* rowp = sb + lane * 128;
#pragma unroll
          for (int j = 0; j < 8; ++j)
            *reinterpret_cast<uint4*>(rowp + ((j ^ (lane & 7)) << 4)) =
                make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
          fence_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(map, sb, col, row0);
            bulk_commit();
          }
          ebuf ^= 1;
        };
        auto load_pack = [&](int col, uint32_t (&w)[32]) {
          uint32_t v0[32], v1[32];
          tmem_ld32(acc + col, v0);
          tmem_ld32(acc + col + 32, v1);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            w[i] = pack_bf16x2(__uint_as_float(v0[2 * i]) * p.alpha, __uint_as_float(v0[2 * i + 1]) * p.alpha);
            w[16 + i] = pack_bf16x2(__uint_as_float(v1[2 * i]) * p.alpha, __uint_as_float(v1[2 * i + 1]) * p.alpha);
          }
        };
        // feature chunk k: gate columns [64 k, 64 k + 64), up columns [128 + 64 k, ...)
#pragma unroll 1
        for (int k = 0; k < 2; ++k) {
          const int f0 = nf0 + k * 64;
          if (row0 >= p.M || f0 >= p.glu_f) continue;   // warp-uniform; glu_f is a multiple of 64
          uint32_t gw[32], uw[32];
          load_pack(k * 64, gw);
          stage_store(gw, &tmD, f0);
          load_pack(128 + k * 64, uw);
          stage_store(uw, &tmD, p.glu_f + f0);
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float2 g2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&gw[i]));
            const float2 u2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&uw[i]));
            gw[i] = pack_bf16x2(__fdividef(g2.x, 1.f + __expf(-g2.x)) * u2.x,
                                __fdividef(g2.y, 1.f + __expf(-g2.y)) * u2.y);
          }
          stage_store(gw, &tmE, f0);
        }
        continue;
      }
      // Chunks of 128 B per row (32 fp32 / 64 bf16 columns): scale (+ beta * C, C fetched by
      // TMA into the staging tile), write the warp's 32 x 128 B tile in the 128B-swizzled layout
      // and TMA-store it (clipped at the matrix edge by the tensor map); two staging buffers
      // per warp so the next chunk fills while the previous store drains.
      const int esz = p.d_fp32 ? 4 : 2;
      const int cc = 128 / esz;                       // columns per chunk
      const int row0 = m0 + h * 128 + q * 32;         // the warp's first row
      const bool use_c = p.C != nullptr && p.beta != 0.f;
#pragma unroll 1
      for (int ch = 0; ch < BN / cc; ++ch) {
        uint32_t v0[32], v1[32];
        tmem_ld32(acc + ch * cc, v0);
        if (esz == 2) tmem_ld32(acc + ch * cc + 32, v1);
        tmem_wait_ld();
        const int col0 = n0 + ch * cc;
        if (row0 >= p.M || col0 >= p.N) continue;     // warp-uniform
        unsigned char* sb = epi + q * 8192 + ebuf * 4096;
        if (lane == 0) bulk_wait_read1();             // the store issued from sb two chunks ago has read it
        __syncwarp();
        if (use_c) {
          if (lane == 0) {
            mbar_expect_tx(&cbar[q * 2 + ebuf], 4096);
            tma_load_2d(sb, &tmC, &cbar[q * 2 + ebuf], col0, row0);
          }
          mbar_wait(&cbar[q * 2 + ebuf], cpar[ebuf], p.err, 107);
          cpar[ebuf] ^= 1;
        }
        unsigned char* rowp = sb + lane * 128;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float4* cp = reinterpret_cast<float4*>(rowp + ((j ^ (lane & 7)) << 4));
          if (esz == 4) {
            float4 o = make_float4(__uint_as_float(v0[4 * j]) * p.alpha, __uint_as_float(v0[4 * j + 1]) * p.alpha,
                                   __uint_as_float(v0[4 * j + 2]) * p.alpha, __uint_as_float(v0[4 * j + 3]) * p.alpha);
            if (use_c) {
              const float4 cv = *cp;
              o.x += p.beta * cv.x; o.y += p.beta * cv.y; o.z += p.beta * cv.z; o.w += p.beta * cv.w;
            }
            *cp = o;
          } else {
            float o[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) o[e] = __uint_as_float(j < 4 ? v0[8 * j + e] : v1[8 * (j - 4) + e]) * p.alpha;
            if (use_c) {
              float cv[8];
              load8(reinterpret_cast<const bf16*>(cp), cv);
#pragma unroll
              for (int e = 0; e < 8; ++e) o[e] += p.beta * cv[e];
            }
            store8(reinterpret_cast<bf16*>(cp), o);
          }
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&tmD, sb, col0, row0);
          bulk_commit();
        }
        ebuf ^= 1;
      }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[ab]);
    }
    if (lane == 0) bulk_wait_all();                   // every store of this warp has landed
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
  if (p.ar_world > 1 && threadIdx.x == 0) {         // the last CTA of the call advances the counter
    __threadfence();
    if (atomicAdd(p.ar_done, 1u) == gridDim.x - 1) {
      *p.ar_done = 0u;
      *p.ar_ctr = *reinterpret_cast<volatile unsigned*>(p.ar_ctr) + 1u;
      __threadfence();
    }
  }
}

// D = alpha * sum_s ws[s] + beta * C   (split-K reduction; one thread per 4 columns)
__global__ void splitk_reduce_kernel(const float* ws, int splits, int M, int N, float alpha, float beta,
                                     const void* C, int64_t ldc, void* D, int64_t ldd, int d_fp32) {
  const int64_t n4 = (int64_t)M * ((N + 3) / 4);
  for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < n4; g += (int64_t)gridDim.x * blockDim.x) {
    const int row = (int)(g / ((N + 3) / 4)), c0 = (int)(g % ((N + 3) / 4)) * 4;
    for (int c = c0; c < c0 + 4 && c < N; ++c) {
      float acc = 0.f;
      for (int sidx = 0; sidx < splits; ++sidx) acc += ws[((int64_t)sidx * M + row) * N + c];
      acc *= alpha;
      if (d_fp32) {
        if (C != nullptr && beta != 0.f) acc += beta * reinterpret_cast<const float*>(C)[(int64_t)row * ldc + c];
        reinterpret_cast<float*>(D)[(int64_t)row * ldd + c] = acc;
      } else {
        if (C != nullptr && beta != 0.f)
          acc += beta * __bfloat162float(reinterpret_cast<const bf16*>(C)[(int64_t)row * ldc + c]);
        reinterpret_cast<bf16*>(D)[(int64_t)row * ldd + c] = __float2bfloat16(acc);
      }
    }
  }
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
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

// Epilogue map over D or C: [rows, cols] row-major (bf16 or fp32), box {128 B of columns, 32 rows},
// 128B swizzle (the staging layout the epilogue writes).
static bool make_epi_map(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int64_t ld, bool fp32) {
  auto fn = encode_fn();
  if (!fn) return false;
  const int esz = fp32 ? 4 : 2;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * esz};
  cuuint32_t box[2] = {(cuuint32_t)(128 / esz), 32};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, fp32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base),
            dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2-D bf16 map over a row-major [rows, cols] matrix with leading dimension ld; box {64, box_rows}.
static bool make_map(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Device word the GEMM's bounded waits report into (allocated once per process).
static int* err_word() {
  static int* w = nullptr;
  if (!w && cudaMalloc(&w, sizeof(int)) == cudaSuccess) cudaMemset(w, 0, sizeof(int));
  return w;
}

}  // namespace gemm100

// Tile height (128 or 256 rows) by estimated time: the persistent CTAs take ceil(tiles / SMs) tiles
// each, and a 128 x 256 tile costs about 0.56 of a 256 x 256 one (half the FLOPs, at ~0.8 instead of
// ~0.9 of the tensor peak: each B slice feeds one MMA instead of two).  So 4032 x 2560 (160 tiles
// of 256 rows = two waves, the second 8 % full) takes 128-row tiles (320 = three full-ish waves),
// while every training shape keeps 256-row tiles.
static int pick_mh(int M, int ntn, int sm_count) {
  const int64_t t2 = (int64_t)((M + 255) / 256) * ntn, t1 = (int64_t)((M + 127) / 128) * ntn;
  const int64_t w2 = (t2 + sm_count - 1) / sm_count, w1 = (t1 + sm_count - 1) / sm_count;
  return 100 * w2 <= 56 * w1 ? 2 : 1;
}

int gemm_splitk(int M, int N, int K, int sm_count) {
  using namespace gemm100;
  const int tiles = ((M + 127) / 128) * ((N + BN - 1) / BN);
  const int kb = (K + BK - 1) / BK;
  if (2 * tiles > sm_count || kb < 8) return 1;
  int splits = sm_count / tiles;
  if (splits > kb / 4) splits = kb / 4;
  if (splits < 2) return 1;
  const int kb_per = (kb + splits - 1) / splits;
  return (kb + kb_per - 1) / kb_per;
}

template <int MH>
static int launch(const CUtensorMap& mA, const CUtensorMap& mB, const CUtensorMap& mD, const CUtensorMap& mC,
                  const CUtensorMap& mE, const gemm100::Params& p, int sm_count, cudaStream_t stream) {
  using namespace gemm100;
  static bool init = false;
  if (!init) {
    cudaFuncSetAttribute(gemm_kernel<MH>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<MH>::SMEM_BYTES);
    init = true;
  }
  const int nt = p.glu_f > 0 ? (p.glu_f + 127) / 128 : (p.N + BN - 1) / BN;
  const int units = ((p.M + Cfg<MH>::BM - 1) / Cfg<MH>::BM) * nt * p.splits;
  const int grid = units < sm_count ? units : sm_count;
  gemm_kernel<MH><<<grid, NTHREADS, Cfg<MH>::SMEM_BYTES, stream>>>(mA, mB, mD, mC, mE, p);
  return 0;
}

int gemm_bf16(GemmLayout layout, bool d_fp32, const GemmArgs& a, int tile, int sm_count, cudaStream_t stream,
              int splits, float* ws) {
  using namespace gemm100;
  if (a.batch != 1) return -20;
  // tile 1: 128 x 256 tiles; tile 2: 256 x 256; otherwise by estimated time (pick_mh)
  const int mh = tile == 1 ? 1 : tile == 2 ? 2 : (splits == 1 ? pick_mh(a.M, (a.N + BN - 1) / BN, sm_count) : 1);
  const int BM = 128 * mh;
  if (a.batch != 1) return -20;
  if (splits < 1 || (splits > 1 && ws == nullptr)) return -21;
  Params p;
  p.M = a.M; p.N = a.N; p.K = a.K;
  p.D = a.D; p.ldd = a.ldd; p.C = a.C; p.ldc = a.ldc;
  p.alpha = a.alpha; p.beta = a.beta; p.d_fp32 = d_fp32 ? 1 : 0;
  p.err = err_word();
  p.glu_f = 0;
  p.ar_world = 1; p.ar_rank = 0; p.ar_tiles_cap = 0; p.ar_mcap = 0;
  p.ar_ctr = nullptr; p.ar_done = nullptr; p.ar_ws = nullptr; p.ar_tile_ctr = nullptr;
  for (int i = 0; i < 8; ++i) { p.ar_recv[i] = nullptr; p.ar_flag[i] = nullptr; }
  p.am_val = nullptr; p.am_idx = nullptr; p.am_ld = 0;
  const int kb = (a.K + BK - 1) / BK;
  p.kb_per = (kb + splits - 1) / splits;
  p.splits = (kb + p.kb_per - 1) / p.kb_per;
  p.ws = ws;
  CUtensorMap mA, mB;
  bool ok;
  switch (layout) {
    case GemmLayout::TN:   // A [M,K] K-major, B [N,K] K-major
      p.a_kmajor = 1; p.b_kmajor = 1;
      ok = make_map(&mA, a.A, a.M, a.K, a.lda, BM) && make_map(&mB, a.B, a.N, a.K, a.ldb, BN);
      break;
    case GemmLayout::TT:   // A [M,K] K-major, B [K,N] N-major
      p.a_kmajor = 1; p.b_kmajor = 0;
      ok = make_map(&mA, a.A, a.M, a.K, a.lda, BM) && make_map(&mB, a.B, a.K, a.N, a.ldb, BK);
      break;
    case GemmLayout::NT:   // A [K,M] M-major, B [K,N] N-major
      p.a_kmajor = 0; p.b_kmajor = 0;
      ok = make_map(&mA, a.A, a.K, a.M, a.lda, BK) && make_map(&mB, a.B, a.K, a.N, a.ldb, BK);
      break;
    default:
      return -11;
  }
  if (!ok) return -12;
  CUtensorMap mD, mC;
  if (!make_epi_map(&mD, a.D, a.M, a.N, a.ldd, d_fp32)) return -14;
  if (a.C != nullptr && a.beta != 0.f) {
    if (!make_epi_map(&mC, a.C, a.M, a.N, a.ldc, d_fp32)) return -15;
  } else {
    mC = mD;
  }
  if (mh == 2) launch<2>(mA, mB, mD, mC, mD, p, sm_count, stream);
  else launch<1>(mA, mB, mD, mC, mD, p, sm_count, stream);
  if (p.splits > 1) {
    const int64_t n4 = (int64_t)a.M * ((a.N + 3) / 4);
    const int blocks = (int)std::min<int64_t>((n4 + 255) / 256, (int64_t)sm_count * 8);
    splitk_reduce_kernel<<<blocks, 256, 0, stream>>>(ws, p.splits, a.M, a.N, a.alpha, a.beta, a.C, a.ldc, a.D, a.ldd,
                                                    p.d_fp32);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -13;
}

int gemm_bf16_allreduce(const GemmArgs& a, const GemmAllreduce& ar, int sm_count, cudaStream_t stream) {
  using namespace gemm100;
  if (ar.world < 2 || ar.world > 8 || ar.rank < 0 || ar.rank >= ar.world) return -30;
  if (a.N % 64 != 0 || a.M > ar.mcap) return -31;
  const int tiles = ((a.M + 127) / 128) * ((a.N + BN - 1) / BN);
  if (tiles > ar.tiles_cap) return -32;
  Params p;
  p.M = a.M; p.N = a.N; p.K = a.K;
  p.D = a.D; p.ldd = a.ldd; p.C = a.C; p.ldc = a.ldc;
  p.alpha = a.alpha; p.beta = a.beta; p.d_fp32 = 0;
  p.err = err_word();
  p.glu_f = 0;
  p.am_val = nullptr; p.am_idx = nullptr; p.am_ld = 0;
  // skinny products split K over otherwise idle SMs; the split partials are summed by the last
  // arriving CTA of each tile before the exchange (workspace: ws_units tiles of 128 x 256 fp32)
  const int kb = (a.K + BK - 1) / BK;
  int splits = (ar.ws != nullptr && ar.tile_ctr != nullptr) ? gemm_splitk(a.M, a.N, a.K, sm_count) : 1;
  while (splits > 1 && (int64_t)tiles * splits > ar.ws_units) --splits;
  p.kb_per = (kb + splits - 1) / splits;
  p.splits = (kb + p.kb_per - 1) / p.kb_per;
  p.ws = nullptr;
  p.a_kmajor = 1; p.b_kmajor = 1;
  p.ar_world = ar.world; p.ar_rank = ar.rank; p.ar_tiles_cap = ar.tiles_cap; p.ar_mcap = ar.mcap;
  p.ar_ctr = ar.ctr; p.ar_done = ar.done; p.ar_ws = ar.ws; p.ar_tile_ctr = ar.tile_ctr;
  for (int i = 0; i < 8; ++i) {
    p.ar_recv[i] = i < ar.world ? reinterpret_cast<bf16*>(ar.recv[i]) : nullptr;
    p.ar_flag[i] = i < ar.world ? ar.flags[i] : nullptr;
  }
  CUtensorMap mA, mB, mD, mC;
  if (!make_map(&mA, a.A, a.M, a.K, a.lda, 128) || !make_map(&mB, a.B, a.N, a.K, a.ldb, BN)) return -12;
  if (!make_epi_map(&mD, a.D, a.M, a.N, a.ldd, false)) return -14;
  if (a.C != nullptr && a.beta != 0.f) {
    if (!make_epi_map(&mC, a.C, a.M, a.N, a.ldc, false)) return -15;
  } else {
    mC = mD;
  }
  launch<1>(mA, mB, mD, mC, mD, p, sm_count, stream);
  return cudaGetLastError() == cudaSuccess ? 0 : -13;
}

int gemm_bf16_swiglu(const GemmArgs& a, void* act, int64_t ld_act, int F, int tile, int sm_count,
                     cudaStream_t stream) {
  using namespace gemm100;
  if (a.batch != 1 || F <= 0 || F % 64 != 0 || a.N != 2 * F) return -40;
  if (a.C != nullptr && a.beta != 0.f) return -41;
  const int mh = tile == 1 ? 1 : tile == 2 ? 2 : pick_mh(a.M, (F + 127) / 128, sm_count);
  Params p;
  p.M = a.M; p.N = a.N; p.K = a.K;
  p.D = a.D; p.ldd = a.ldd; p.C = nullptr; p.ldc = a.ldd;
  p.alpha = a.alpha; p.beta = 0.f; p.d_fp32 = 0;
  p.err = err_word();
  p.glu_f = F;
  p.am_val = nullptr; p.am_idx = nullptr; p.am_ld = 0;
  p.ar_world = 1; p.ar_rank = 0; p.ar_tiles_cap = 0; p.ar_mcap = 0;
  p.ar_ctr = nullptr; p.ar_done = nullptr; p.ar_ws = nullptr; p.ar_tile_ctr = nullptr;
  for (int i = 0; i < 8; ++i) { p.ar_recv[i] = nullptr; p.ar_flag[i] = nullptr; }
  const int kb = (a.K + BK - 1) / BK;
  p.splits = 1; p.kb_per = kb; p.ws = nullptr;
  p.a_kmajor = 1; p.b_kmajor = 1;
  CUtensorMap mA, mB, mD, mE;
  if (!make_map(&mA, a.A, a.M, a.K, a.lda, 128 * mh) || !make_map(&mB, a.B, a.N, a.K, a.ldb, 128)) return -12;
  if (!make_epi_map(&mD, a.D, a.M, a.N, a.ldd, false) || !make_epi_map(&mE, act, a.M, F, ld_act, false)) return -14;
  if (mh == 2) launch<2>(mA, mB, mD, mD, mE, p, sm_count, stream);
  else launch<1>(mA, mB, mD, mD, mE, p, sm_count, stream);
  return cudaGetLastError() == cudaSuccess ? 0 : -13;
}

namespace gemm100 {
// Greedy tokens from the argmax epilogue's per-tile partials: one warp per row, first index on ties.
__global__ void argmax_tiles_kernel(const float* __restrict__ val, const int* __restrict__ idx, int M, int nt,
                                    int64_t* __restrict__ out) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= M) return;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int t = lane; t < nt; t += 32) {
    const float v = val[(int64_t)row * nt + t];
    const int i = idx[(int64_t)row * nt + t];
    if (v > best || (v == best && i < bi)) {
      best = v;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float v2 = __shfl_xor_sync(0xffffffffu, best, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
    if (v2 > best || (v2 == best && i2 < bi)) {
      best = v2;
      bi = i2;
    }
  }
  if (lane == 0) out[row] = bi;
}
}  // namespace gemm100

int gemm_argmax_tiles(int N) { return (N + gemm100::BN - 1) / gemm100::BN; }

int gemm_bf16_argmax(const GemmArgs& a, float* am_val, int* am_idx, int64_t* out, int sm_count, cudaStream_t stream) {
  using namespace gemm100;
  if (a.batch != 1) return -20;
  const int mh = pick_mh(a.M, (a.N + BN - 1) / BN, sm_count);
  Params p;
  p.M = a.M; p.N = a.N; p.K = a.K;
  p.D = am_val; p.ldd = 0; p.C = nullptr; p.ldc = 0;
  p.alpha = 1.f; p.beta = 0.f; p.d_fp32 = 1;
  p.err = err_word();
  p.glu_f = 0;
  p.ar_world = 1; p.ar_rank = 0; p.ar_tiles_cap = 0; p.ar_mcap = 0;
  p.ar_ctr = nullptr; p.ar_done = nullptr; p.ar_ws = nullptr; p.ar_tile_ctr = nullptr;
  for (int i = 0; i < 8; ++i) { p.ar_recv[i] = nullptr; p.ar_flag[i] = nullptr; }
  const int nt = (a.N + BN - 1) / BN;
  p.am_val = am_val; p.am_idx = am_idx; p.am_ld = nt;
  const int kb = (a.K + BK - 1) / BK;
  p.splits = 1; p.kb_per = kb; p.ws = nullptr;
  p.a_kmajor = 1; p.b_kmajor = 1;
  CUtensorMap mA, mB, mD;
  if (!make_map(&mA, a.A, a.M, a.K, a.lda, 128 * mh) || !make_map(&mB, a.B, a.N, a.K, a.ldb, BN)) return -12;
  // D is never written in argmax mode; the epilogue map only has to be a valid descriptor (A's)
  if (!make_map(&mD, a.A, a.M, a.K, a.lda, 32)) return -14;
  if (mh == 2) launch<2>(mA, mB, mD, mD, mD, p, sm_count, stream);
  else launch<1>(mA, mB, mD, mD, mD, p, sm_count, stream);
  argmax_tiles_kernel<<<(a.M + 7) / 8, 256, 0, stream>>>(am_val, am_idx, a.M, nt, out);
  return cudaGetLastError() == cudaSuccess ? 0 : -13;
}

int* gemm_error_word() { return gemm100::err_word(); }

}  // namespace trida
