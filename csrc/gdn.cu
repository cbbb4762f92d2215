// Gated-delta-rule (GDN) linear attention for the hybrid decoder (sm_100a).
//
// Behaviour follows the reference's hybrid layers: train/models/hybrid.py:215-324 (two-stream
// recurrence: a causal pass over the clean stream, then every noisy block of every view restarted
// from the clean state at the end of the previous block and read out at its own block end),
// :137-212 (causal gated-delta rule with per-document resets), :327-451 (short depthwise conv +
// SiLU, two-stream variant whose in-block taps read the noisy stream).
//
// Recurrence per value head (state S [dk=128, dv=128] in fp32; q, k L2-normalised, q * dk^-0.5):
//     S' = exp(g) S ;  u = beta (v - S'^T k) ;  S = S' + k u^T ;  o = S^T q
// Every value column of S evolves on its own, so a head is split over 8 CTAs of 16 columns and a
// CTA keeps its 128 x 16 slice in registers: thread (column c, row part r) owns 16 rows of column
// c (4 groups of 4, interleaved so shared-memory reads are conflict-free); the dot products over
// dk are 3-step shuffles inside each group of 8 lanes.
//
// Forward: fwd_clean walks the clean stream (or the whole causal row) in chunks, storing the state
// at every chunk start (block starts in the two-stream layout) as the backward's checkpoints and
// the noisy blocks' initial states; fwd_noisy runs every (block, view) of the noisy streams in
// parallel from those states.
// Backward: per chunk, recompute forward from the checkpoint with sub-checkpoints every SUB tokens,
// then replay each sub-chunk keeping S' in registers and sweep it in reverse.  Gradients w.r.t. q
// and k are sums over the 128 value columns: reduced across the 4 columns of a warp by shuffles
// and across the CTA's 4 warps in shared memory; each CTA then writes its partial rows (dq | dk |
// dbeta | dg per token) to a global buffer with plain coalesced stores, and the closing pass sums
// the head's 8 column groups (no inter-CTA synchronisation on the sequential path).
#include "common.cuh"
#include "ops.h"

namespace trida {
namespace gdn {

constexpr int DK = 128, DV = 128;
constexpr int CG = 16;          // value columns per CTA
constexpr int NCG = DV / CG;    // CTAs per head
constexpr int RP = 8;           // threads per column
constexpr int RPT = DK / RP;    // rows per thread
constexpr int NT = CG * RP;     // 128 threads
constexpr int SUB = 4;          // backward replay sub-chunk
constexpr int RED = 2 * DK + 4; // per-token reduction row: dq | dk | dbeta | dg (16-byte rows)
constexpr int MAXCH = 64;

struct Args {
  int B, T, Hk, Hv;
  int mode;                 // 0 causal, 1 two-stream
  int L, V, bd;             // two-stream geometry
  int causal_clean, causal_noisy;
  int ch, nch;              // clean-stream chunk length and count
  const uint8_t* doc;       // [B, Lc] document-start flags of the clean stream (may be null)
  const bf16* mixed;        // [B*T, ldm]: q | k | v (conv output)
  int64_t ldm;
  const bf16* ga;           // gate pre-activation a [B*T, Hv] (row stride ldg)
  const bf16* gb;           // gate pre-activation b
  int64_t ldg;
  const float* A_log;
  const float* dt_bias;
  float scale;
  float* ckpt;              // [B, Hv, nch, NCG, RPT, NT]
  bf16* o;                  // [B*T, Hv*DV]
  const bf16* d_o;          // [B*T, Hv*DV]
  float* dpart;             // [B*T, Hv, NCG, RED] per-CTA partial rows: dq | dk | dbeta | dg
  bf16* dv;                 // v-gradient rows [B*T, lddv] (head columns at hv*DV)
  int64_t lddv;
  float* dinit;             // [B, Hv, nch, NCG, RPT, NT]
  float* final_state;       // optional [B, Hv, DK, DV] state after the last clean token (serving prefill)
  const float* qk;          // prep: [B*T, Hk, 2, DK] L2-normalised q (times scale) and k
  const float* ab;          // prep: [B*T, Hv, 2] decay exp(g) and beta
};

struct Stage {
  float* q;     // [ch][DK]
  float* k;     // [ch][DK]
  float* v;     // [ch][CG]
  float* dO;    // [ch][CG]
  float* al;    // [ch]
  float* be;    // [ch]
  float* ob;    // [ch][CG]  (forward output staging / backward dv staging)
  int* rs;      // [ch]
  float* sck;   // [ch/SUB][RPT][NT] (backward sub-checkpoints)
  float* red;   // [SUB][RED]        (backward reduction rows)
};

__host__ __device__ inline size_t stage_floats(int ch, bool bwd) {
  size_t n = (size_t)ch * (2 * DK + 3 * CG + 3);
  if (bwd) n += (size_t)((ch + SUB - 1) / SUB) * RPT * NT + SUB * RED;
  return n;
}

__device__ inline Stage carve(float* sm, int ch, bool bwd) {
  Stage s;
  s.q = sm; sm += ch * DK;
  s.k = sm; sm += ch * DK;
  s.v = sm; sm += ch * CG;
  s.dO = sm; sm += ch * CG;
  s.ob = sm; sm += ch * CG;
  s.al = sm; sm += ch;
  s.be = sm; sm += ch;
  s.rs = reinterpret_cast<int*>(sm); sm += ch;
  if (bwd) {
    s.sck = sm; sm += ((ch + SUB - 1) / SUB) * RPT * NT;
    s.red = sm;
  }
  return s;
}

__device__ __forceinline__ float rsum8(float x) {
  x += __shfl_xor_sync(0xffffffffu, x, 1);
  x += __shfl_xor_sync(0xffffffffu, x, 2);
  x += __shfl_xor_sync(0xffffffffu, x, 4);
  return x;
}

__device__ __forceinline__ float softplus_f(float x) { return x > 20.f ? x : log1pf(expf(x)); }

// Thread (column, row part rp) owns rows {32 f + 4 rp + e : f, e in 0..3} of its column, so the 8
// row parts of a warp read one contiguous 128 B line of a staged q / k vector per float4 load
// (conflict-free).  `p` points at the vector plus 4 rp.
__device__ __forceinline__ int own_row(int rp, int i) { return (i >> 2) * 32 + rp * 4 + (i & 3); }

__device__ __forceinline__ void load16(const float* p, float (&x)[RPT]) {
#pragma unroll
  for (int i = 0; i < RPT; i += 4) {
    const float4 t = *reinterpret_cast<const float4*>(p + (i >> 2) * 32);
    x[i] = t.x; x[i + 1] = t.y; x[i + 2] = t.z; x[i + 3] = t.w;
  }
}

// One recurrence step on the thread's slice; returns u (column scalar) and v - p.
__device__ __forceinline__ void fwd_step(float (&S)[RPT], const float* kp, float al, float be, float vc, float& u,
                                         float& vmp) {
  float k[RPT];
  load16(kp, k);
  float a0 = 0.f, a1 = 0.f;
#pragma unroll
  for (int i = 0; i < RPT; i += 2) {
    a0 = fmaf(S[i], k[i], a0);
    a1 = fmaf(S[i + 1], k[i + 1], a1);
  }
  const float p = al * rsum8(a0 + a1);
  vmp = vc - p;
  u = be * vmp;
#pragma unroll
  for (int i = 0; i < RPT; ++i) S[i] = fmaf(al, S[i], k[i] * u);
}

__device__ __forceinline__ float readout(const float (&S)[RPT], const float* qp) {
  float q[RPT];
  load16(qp, q);
  float a0 = 0.f, a1 = 0.f;
#pragma unroll
  for (int i = 0; i < RPT; i += 2) {
    a0 = fmaf(S[i], q[i], a0);
    a1 = fmaf(S[i + 1], q[i + 1], a1);
  }
  return rsum8(a0 + a1);
}

__device__ __forceinline__ void store_o(const Args& a, const Stage& s, int b, int hv, int cg, int tok0, int n) {
  for (int idx = threadIdx.x; idx < n * CG; idx += NT) {
    const int j = idx / CG, c = idx % CG;
    a.o[((int64_t)b * a.T + tok0 + j) * (a.Hv * DV) + hv * DV + cg * CG + c] = __float2bfloat16(s.ob[idx]);
  }
}

__device__ __forceinline__ float* state_ptr(float* base, const Args& a, int b, int hv, int c, int cg) {
  return base + ((((int64_t)b * a.Hv + hv) * a.nch + c) * NCG + cg) * (RPT * NT);
}

// ---------------------------------------------------------------------------------------------
// prep: per token and key head the L2-normalised q (times scale) and k, per value head the decay
// exp(g) and beta, computed once (fully parallel) so the sequential scans stage plain copies.
// ---------------------------------------------------------------------------------------------
__global__ void prep_kernel(const Args a, float* qk, float* ab, int rows) {
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int per_row = 2 * a.Hk + 1;                 // q / k per key head, then one warp for the gates
  if (gw >= (int64_t)rows * per_row) return;
  const int64_t row = gw / per_row;
  const int w = (int)(gw % per_row);
  if (w < 2 * a.Hk) {
    const int hk = w >> 1, isk = w & 1;
    const bf16* src = a.mixed + row * a.ldm + isk * a.Hk * DK + hk * DK + lane * 4;
    const uint2 raw = *reinterpret_cast<const uint2*>(src);
    const bf16* e = reinterpret_cast<const bf16*>(&raw);
    float v[4], ss = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[i] = __bfloat162float(e[i]);
      ss += v[i] * v[i];
    }
    ss = warp_sum(ss);
    const float r = rsqrtf(ss + 1e-6f) * (isk ? 1.f : a.scale);
    *reinterpret_cast<float4*>(qk + ((row * a.Hk + hk) * 2 + isk) * DK + lane * 4) =
        make_float4(v[0] * r, v[1] * r, v[2] * r, v[3] * r);
  } else {
    for (int h = lane; h < a.Hv; h += 32) {
      const float av = __bfloat162float(a.ga[row * a.ldg + h]) + a.dt_bias[h];
      const float bv = __bfloat162float(a.gb[row * a.ldg + h]);
      ab[(row * a.Hv + h) * 2] = expf(-expf(a.A_log[h]) * softplus_f(av));
      ab[(row * a.Hv + h) * 2 + 1] = 1.f / (1.f + expf(-bv));
    }
  }
}

// Stage n tokens (row-relative tok0 ..) of row b from the prep buffers: plain coalesced copies of
// the normalised q / k, the CTA's v (and dO) columns, decay / beta and the reset flags (clean
// positions pos0.. when pos0 >= 0).
__device__ __forceinline__ void stage_prepped(const Args& a, const Stage& s, const float* qk, const float* ab, int b,
                                              int hv, int cg, int tok0, int n, int pos0, bool bwd) {
  const int hk = hv / (a.Hv / a.Hk);
  const int Lc = a.mode ? a.L : a.T;
  for (int idx = threadIdx.x; idx < n * (DK / 4) * 2; idx += NT) {
    const int j = idx / (DK / 2), rem = idx % (DK / 2), isk = rem / (DK / 4), c4 = rem % (DK / 4);
    const int64_t row = (int64_t)b * a.T + tok0 + j;
    const float4 v = *reinterpret_cast<const float4*>(qk + ((row * a.Hk + hk) * 2 + isk) * DK + c4 * 4);
    *reinterpret_cast<float4*>((isk ? s.k : s.q) + j * DK + c4 * 4) = v;
  }
  for (int idx = threadIdx.x; idx < n * CG; idx += NT) {
    const int j = idx / CG, c = idx % CG;
    const int64_t row = (int64_t)b * a.T + tok0 + j;
    s.v[idx] = __bfloat162float(a.mixed[row * a.ldm + 2 * a.Hk * DK + hv * DV + cg * CG + c]);
    if (bwd) s.dO[idx] = __bfloat162float(a.d_o[row * (int64_t)(a.Hv * DV) + hv * DV + cg * CG + c]);
  }
  for (int j = threadIdx.x; j < n; j += NT) {
    const int64_t row = (int64_t)b * a.T + tok0 + j;
    s.al[j] = ab[(row * a.Hv + hv) * 2];
    s.be[j] = ab[(row * a.Hv + hv) * 2 + 1];
    s.rs[j] = (pos0 >= 0 && a.doc != nullptr) ? (int)a.doc[(int64_t)b * Lc + pos0 + j] : 0;
  }
}

// ---------------------------------------------------------------------------------------------
// forward
// ---------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(NT) fwd_clean_kernel(const Args a) {
  extern __shared__ float smem[];
  const int cg = blockIdx.x, hv = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, col = tid / RP, rp = tid % RP;
  const Stage s = carve(smem, a.ch, false);
  const int Lc = a.mode ? a.L : a.T;
  const bool tok_read = a.mode == 0 || a.causal_clean;
  float S[RPT];
#pragma unroll
  for (int i = 0; i < RPT; ++i) S[i] = 0.f;
  for (int c = 0; c < a.nch; ++c) {
    const int p0 = c * a.ch, n = min(a.ch, Lc - p0);
    float* ck = state_ptr(a.ckpt, a, b, hv, c, cg);
#pragma unroll
    for (int i = 0; i < RPT; ++i) ck[i * NT + tid] = S[i];
    stage_prepped(a, s, a.qk, a.ab, b, hv, cg, p0, n, p0, false);
    __syncthreads();
    for (int j = 0; j < n; ++j) {
      if (s.rs[j]) {
#pragma unroll
        for (int i = 0; i < RPT; ++i) S[i] = 0.f;
      }
      float u, vmp;
      fwd_step(S, s.k + j * DK + rp * 4, s.al[j], s.be[j], s.v[j * CG + col], u, vmp);
      if (tok_read) {
        const float o = readout(S, s.q + j * DK + rp * 4);
        if (rp == 0) s.ob[j * CG + col] = o;
      }
    }
    if (!tok_read) {
      for (int j = 0; j < n; ++j) {
        const float o = readout(S, s.q + j * DK + rp * 4);
        if (rp == 0) s.ob[j * CG + col] = o;
      }
    }
    __syncthreads();
    store_o(a, s, b, hv, cg, p0, n);
    __syncthreads();
  }
  if (a.final_state != nullptr) {
    float* f = a.final_state + ((int64_t)b * a.Hv + hv) * DK * DV + cg * CG + col;
#pragma unroll
    for (int i = 0; i < RPT; ++i) f[own_row(rp, i) * DV] = S[i];
  }
}

// ---------------------------------------------------------------------------------------------
// serving: one canvas of T rows per request from the cached state (rows < n_clean token-causal,
// the rest read the state after the last row), and the commit that advances the cached state by
// adv[b] rows.  The state cache is kept in the thread-native layout [slots, Hv, NCG, RPT, NT] so
// every load / store is coalesced; a prep pass writes each row's L2-normalised q (times scale) and
// k once ([rows, Hk, 2, DK] fp32) and its decay / beta ([rows, Hv, 2]) for both kernels.
// ---------------------------------------------------------------------------------------------
// Serving canvas / commit with two column groups per CTA (blockIdx.x = group pair): thread (col,
// rp) carries the state slices of column col of both groups, so every k / q slice read from shared
// memory per recurrence step serves two columns, and the two dependency chains interleave.  With
// one group per CTA the kernel was shared-memory bound (each step re-read the k row per column;
// 0.255 -> 0.081 ms for 64 requests x 7 rows).  The cached state keeps the per-group layout
// [Hv][NCG][RPT][NT] of the training kernels; the second group's v and outputs use the stage's
// dO buffer and T * CG floats past the stage.
__device__ __forceinline__ void fwd_step2(float (&S0)[RPT], float (&S1)[RPT], const float* kp, float al, float be,
                                          float v0, float v1) {
  float k[RPT];
  load16(kp, k);
  float a0 = 0.f, a1 = 0.f, c0 = 0.f, c1 = 0.f;
#pragma unroll
  for (int i = 0; i < RPT; i += 2) {
    a0 = fmaf(S0[i], k[i], a0);
    a1 = fmaf(S0[i + 1], k[i + 1], a1);
    c0 = fmaf(S1[i], k[i], c0);
    c1 = fmaf(S1[i + 1], k[i + 1], c1);
  }
  const float u0 = be * (v0 - al * rsum8(a0 + a1));
  const float u1 = be * (v1 - al * rsum8(c0 + c1));
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    S0[i] = fmaf(al, S0[i], k[i] * u0);
    S1[i] = fmaf(al, S1[i], k[i] * u1);
  }
}

__device__ __forceinline__ void readout2(const float (&S0)[RPT], const float (&S1)[RPT], const float* qp, float& o0,
                                         float& o1) {
  float q[RPT];
  load16(qp, q);
  float a0 = 0.f, a1 = 0.f, c0 = 0.f, c1 = 0.f;
#pragma unroll
  for (int i = 0; i < RPT; i += 2) {
    a0 = fmaf(S0[i], q[i], a0);
    a1 = fmaf(S0[i + 1], q[i + 1], a1);
    c0 = fmaf(S1[i], q[i], c0);
    c1 = fmaf(S1[i + 1], q[i + 1], c1);
  }
  o0 = rsum8(a0 + a1);
  o1 = rsum8(c0 + c1);
}

// v of column group cg for rows [tok0, tok0 + n) into dst[n][CG]
__device__ __forceinline__ void stage_v(const Args& a, float* dst, int b, int hv, int cg, int tok0, int n) {
  for (int idx = threadIdx.x; idx < n * CG; idx += NT) {
    const int j = idx / CG, c = idx % CG;
    const int64_t row = (int64_t)b * a.T + tok0 + j;
    dst[idx] = __bfloat162float(a.mixed[row * a.ldm + 2 * a.Hk * DK + hv * DV + cg * CG + c]);
  }
}

// outputs of both groups for rows [tok0, tok0 + n) from the staging buffers
__device__ __forceinline__ void store_o2(const Args& a, const Stage& s, const float* ob1, int b, int hv, int cg,
                                         int tok0, int n) {
  store_o(a, s, b, hv, cg, tok0, n);
  for (int idx = threadIdx.x; idx < n * CG; idx += NT) {
    const int j = idx / CG, c = idx % CG;
    a.o[((int64_t)b * a.T + tok0 + j) * (a.Hv * DV) + hv * DV + (cg + 1) * CG + c] = __float2bfloat16(ob1[idx]);
  }
}

// Rows are staged CANVAS_CHUNK at a time (about 21 KB of shared memory per CTA instead of 81 KB for
// a 63-row canvas), so several CTAs share an SM and hide each other's step latency; the mask rows'
// readouts (from the state after every row) take a second pass over their q rows.
constexpr int CANVAS_CHUNK = 16;
__host__ __device__ inline size_t canvas2_floats(int T) {
  const int ch = T < CANVAS_CHUNK ? T : CANVAS_CHUNK;
  return stage_floats(ch, false) + (size_t)ch * CG;
}

__global__ void __launch_bounds__(NT) canvas2_kernel(const Args a, const float* qk, const float* ab, const float* ssm,
                                                     const int* slot, int n_clean) {
  extern __shared__ float smem[];
  const int cg = 2 * blockIdx.x, hv = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, col = tid / RP, rp = tid % RP;
  const int ch = min(a.T, CANVAS_CHUNK);
  const Stage s = carve(smem, ch, false);
  float* v1 = s.dO;
  float* ob1 = smem + stage_floats(ch, false);
  const float* base = ssm + (((int64_t)slot[b] * a.Hv + hv) * NCG + cg) * (RPT * NT);
  float S0[RPT], S1[RPT];
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    S0[i] = base[i * NT + tid];
    S1[i] = base[RPT * NT + i * NT + tid];
  }
  for (int c0 = 0; c0 < a.T; c0 += ch) {
    const int n = min(ch, a.T - c0);
    __syncthreads();                       // the previous chunk's stage and outputs are consumed
    stage_prepped(a, s, qk, ab, b, hv, cg, c0, n, -1, false);
    stage_v(a, v1, b, hv, cg + 1, c0, n);
    __syncthreads();
    for (int j = 0; j < n; ++j) {
      fwd_step2(S0, S1, s.k + j * DK + rp * 4, s.al[j], s.be[j], s.v[j * CG + col], v1[j * CG + col]);
      if (c0 + j < n_clean) {
        float o0, o1;
        readout2(S0, S1, s.q + j * DK + rp * 4, o0, o1);
        if (rp == 0) {
          s.ob[j * CG + col] = o0;
          ob1[j * CG + col] = o1;
        }
      }
    }
    __syncthreads();
    const int nout = min(n, n_clean - c0);
    if (nout > 0) store_o2(a, s, ob1, b, hv, cg, c0, nout);
  }
  const bool single = a.T <= ch;          // one chunk: the mask rows' q are still staged
  for (int c0 = max(n_clean, 0); c0 < a.T; c0 += ch) {
    const int n = min(ch, a.T - c0), off = single ? c0 : 0;
    __syncthreads();
    if (!single) {
      stage_prepped(a, s, qk, ab, b, hv, cg, c0, n, -1, false);
      __syncthreads();
    }
    for (int j = 0; j < n; ++j) {
      float o0, o1;
      readout2(S0, S1, s.q + (off + j) * DK + rp * 4, o0, o1);
      if (rp == 0) {
        s.ob[j * CG + col] = o0;
        ob1[j * CG + col] = o1;
      }
    }
    __syncthreads();
    store_o2(a, s, ob1, b, hv, cg, c0, n);
  }
}

__global__ void __launch_bounds__(NT) commit2_kernel(const Args a, const float* qk, const float* ab, float* ssm,
                                                     const int* slot, const int* adv) {
  extern __shared__ float smem[];
  const int cg = 2 * blockIdx.x, hv = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, col = tid / RP, rp = tid % RP;
  const int ch = min(a.T, CANVAS_CHUNK);
  const Stage s = carve(smem, ch, false);
  float* v1 = s.dO;
  const int total = min(adv[b], a.T);
  float* base = ssm + (((int64_t)slot[b] * a.Hv + hv) * NCG + cg) * (RPT * NT);
  float S0[RPT], S1[RPT];
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    S0[i] = base[i * NT + tid];
    S1[i] = base[RPT * NT + i * NT + tid];
  }
  for (int c0 = 0; c0 < total; c0 += ch) {
    const int n = min(ch, total - c0);
    __syncthreads();
    stage_prepped(a, s, qk, ab, b, hv, cg, c0, n, -1, false);
    stage_v(a, v1, b, hv, cg + 1, c0, n);
    __syncthreads();
    for (int j = 0; j < n; ++j)
      fwd_step2(S0, S1, s.k + j * DK + rp * 4, s.al[j], s.be[j], s.v[j * CG + col], v1[j * CG + col]);
  }
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    base[i * NT + tid] = S0[i];
    base[RPT * NT + i * NT + tid] = S1[i];
  }
}

// Initial state of noisy block n of row b: the clean state at the start of block n, zero for the
// first block and at a document start.
__device__ __forceinline__ bool noisy_init(const Args& a, int b, int n) {
  return n > 0 && !(a.doc != nullptr && a.doc[(int64_t)b * a.L + n * a.bd]);
}

__global__ void __launch_bounds__(NT) fwd_noisy_kernel(const Args a) {
  extern __shared__ float smem[];
  const int nb = a.L / a.bd;
  const int cg = blockIdx.x, hv = blockIdx.y, n = blockIdx.z % nb, b = blockIdx.z / nb;
  const int tid = threadIdx.x, col = tid / RP, rp = tid % RP;
  const Stage s = carve(smem, a.bd, false);
  float S0[RPT];
  const bool from_clean = noisy_init(a, b, n);
  const float* ck = state_ptr(a.ckpt, a, b, hv, n, cg);
#pragma unroll
  for (int i = 0; i < RPT; ++i) S0[i] = from_clean ? ck[i * NT + tid] : 0.f;
  for (int v = 0; v < a.V; ++v) {
    const int tok0 = (1 + v) * a.L + n * a.bd;
    stage_prepped(a, s, a.qk, a.ab, b, hv, cg, tok0, a.bd, -1, false);
    __syncthreads();
    float S[RPT];
#pragma unroll
    for (int i = 0; i < RPT; ++i) S[i] = S0[i];
    for (int j = 0; j < a.bd; ++j) {
      float u, vmp;
      fwd_step(S, s.k + j * DK + rp * 4, s.al[j], s.be[j], s.v[j * CG + col], u, vmp);
      if (a.causal_noisy) {
        const float o = readout(S, s.q + j * DK + rp * 4);
        if (rp == 0) s.ob[j * CG + col] = o;
      }
    }
    if (!a.causal_noisy) {
      for (int j = 0; j < a.bd; ++j) {
        const float o = readout(S, s.q + j * DK + rp * 4);
        if (rp == 0) s.ob[j * CG + col] = o;
      }
    }
    __syncthreads();
    store_o(a, s, b, hv, cg, tok0, a.bd);
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------------------------
// backward
// ---------------------------------------------------------------------------------------------
// Sum x[16] (this thread's rows, its column) over the warp's 4 columns and add the 4 resulting
// row sums into dst[row] (shared memory; the CTA's 4 warps add into the same row).
__device__ __forceinline__ void col_reduce_add(const float (&x)[RPT], float* dst, int lane, int rp) {
  const int h1 = (lane >> 4) & 1, h2 = (lane >> 3) & 1;
  float y[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float send = h1 ? x[i] : x[i + 8];
    const float keep = h1 ? x[i + 8] : x[i];
    y[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
  float z[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float send = h2 ? y[i] : y[i + 4];
    const float keep = h2 ? y[i + 4] : y[i];
    z[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
  const int r0 = (2 * h1 + h2) * 32 + rp * 4;   // rows own_row(rp, 8 h1 + 4 h2 + 0..3)
#pragma unroll
  for (int i = 0; i < 4; ++i) atomicAdd(dst + r0 + i, z[i]);
}

struct Ctx {
  int b, hv, cg, tid, col, rp, lane;
  int par;
};

constexpr int FL_DQ = 1, FL_DK = 2, FL_SC = 4;

// Write the CTA's m reduction rows (tokens tok0..) to its slot of the partial buffer: the fields
// selected by `what` only, so the read-out pass (dq) and the sweep (dk, scalars) of one token can
// write at different times.
__device__ void flush(const Args& a, const Stage& s, Ctx& x, int tok0, int m, int what) {
  __syncthreads();
  for (int idx = x.tid; idx < m * (RED / 4); idx += NT) {
    const int t = idx / (RED / 4), f4 = idx % (RED / 4);
    const int e = f4 * 4;
    const bool want = e < DK ? (what & FL_DQ) : e < 2 * DK ? (what & FL_DK) : (what & FL_SC);
    if (!want) continue;
    const int64_t row = (int64_t)x.b * a.T + tok0 + t;
    *reinterpret_cast<float4*>(a.dpart + ((row * a.Hv + x.hv) * NCG + x.cg) * RED + e) =
        *reinterpret_cast<const float4*>(s.red + t * RED + e);
  }
  __syncthreads();
}

__device__ __forceinline__ void zero_red(const Stage& s, const Ctx& x) {
  for (int i = x.tid; i < SUB * RED; i += NT) s.red[i] = 0.f;
  __syncthreads();
}

// Reverse pass over the n staged tokens (row-relative tok0..).  Sst: state entering token 0 (before
// any reset); dS: on entry the gradient w.r.t. the state after the last token, on exit w.r.t. Sst.
// end_read: every token read the state after the last token (block-end read-out).
__device__ void bwd_segment(const Args& a, const Stage& s, Ctx& x, const float (&Sst)[RPT], float (&dS)[RPT], int tok0,
                            int n, bool end_read) {
  const int tid = x.tid, col = x.col, rp = x.rp, lane = x.lane;
  float S[RPT];
#pragma unroll
  for (int i = 0; i < RPT; ++i) S[i] = Sst[i];
  // pass 1: forward with sub-checkpoints
  for (int j = 0; j < n; ++j) {
    if (j % SUB == 0) {
#pragma unroll
      for (int i = 0; i < RPT; ++i) s.sck[((j / SUB) * RPT + i) * NT + tid] = S[i];
    }
    if (s.rs[j]) {
#pragma unroll
      for (int i = 0; i < RPT; ++i) S[i] = 0.f;
    }
    float u, vmp;
    fwd_step(S, s.k + j * DK + rp * 4, s.al[j], s.be[j], s.v[j * CG + col], u, vmp);
  }
  if (end_read) {
    // o_j = S_end^T q_j:  dS_end += sum_j q_j do_j^T ;  dq_j = S_end do_j
    for (int j0 = 0; j0 < n; j0 += SUB) {
      const int m = min(SUB, n - j0);
      zero_red(s, x);
      float* red = s.red;
      for (int t = 0; t < m; ++t) {
        const int j = j0 + t;
        const float doc = s.dO[j * CG + col];
        float q[RPT], dq[RPT];
        load16(s.q + j * DK + rp * 4, q);
#pragma unroll
        for (int i = 0; i < RPT; ++i) {
          dq[i] = S[i] * doc;
          dS[i] = fmaf(q[i], doc, dS[i]);
        }
        col_reduce_add(dq, red + t * RED, lane, rp);
      }
      flush(a, s, x, tok0 + j0, m, FL_DQ);
    }
  }
  // pass 2: replay each sub-chunk (S' in registers) and sweep it in reverse
  const int nsub = (n + SUB - 1) / SUB;
  for (int sc = nsub - 1; sc >= 0; --sc) {
    const int j0 = sc * SUB, m = min(SUB, n - j0);
    zero_red(s, x);
    float* red = s.red;
#pragma unroll
    for (int i = 0; i < RPT; ++i) S[i] = s.sck[(sc * RPT + i) * NT + tid];
    float Sp[SUB][RPT], uu[SUB], vm[SUB];
#pragma unroll
    for (int t = 0; t < SUB; ++t) {
      if (t < m) {
        const int j = j0 + t;
        if (s.rs[j]) {
#pragma unroll
          for (int i = 0; i < RPT; ++i) S[i] = 0.f;
        }
        const float al = s.al[j];
#pragma unroll
        for (int i = 0; i < RPT; ++i) Sp[t][i] = al * S[i];
        fwd_step(S, s.k + j * DK + rp * 4, al, s.be[j], s.v[j * CG + col], uu[t], vm[t]);
      }
    }
#pragma unroll
    for (int t = SUB - 1; t >= 0; --t) {
      if (t < m) {
        const int j = j0 + t;
        const float al = s.al[j], be = s.be[j];
        const float doc = s.dO[j * CG + col];
        float k[RPT], dq[RPT], dk[RPT];
        load16(s.k + j * DK + rp * 4, k);
        if (!end_read) {
          float q[RPT];
          load16(s.q + j * DK + rp * 4, q);
#pragma unroll
          for (int i = 0; i < RPT; ++i) {
            dq[i] = fmaf(k[i], uu[t], Sp[t][i]) * doc;   // S_t = S' + k u^T
            dS[i] = fmaf(q[i], doc, dS[i]);
          }
        }
        float a0 = 0.f, a1 = 0.f;
#pragma unroll
        for (int i = 0; i < RPT; i += 2) {
          a0 = fmaf(dS[i], k[i], a0);
          a1 = fmaf(dS[i + 1], k[i + 1], a1);
        }
        const float du = rsum8(a0 + a1);
        const float dp = -be * du;
        float g0 = 0.f, g1 = 0.f;
#pragma unroll
        for (int i = 0; i < RPT; ++i) {
          dk[i] = dS[i] * uu[t];
          dS[i] = fmaf(k[i], dp, dS[i]);          // gradient w.r.t. S'
          dk[i] = fmaf(Sp[t][i], dp, dk[i]);
          if (i & 1) g1 = fmaf(dS[i], Sp[t][i], g1); else g0 = fmaf(dS[i], Sp[t][i], g0);
          dS[i] *= al;
        }
        if (s.rs[j]) {
#pragma unroll
          for (int i = 0; i < RPT; ++i) dS[i] = 0.f;
        }
        if (rp == 0) s.ob[t * CG + col] = be * du;          // dv
        float* rrow = red + t * RED;
        if (!end_read) col_reduce_add(dq, rrow, lane, rp);
        col_reduce_add(dk, rrow + DK, lane, rp);
        float dbt = du * vm[t];                            // one column's share (same in its 8 lanes)
        dbt += __shfl_xor_sync(0xffffffffu, dbt, 8);
        dbt += __shfl_xor_sync(0xffffffffu, dbt, 16);
        const float dg = warp_sum(g0 + g1);
        if (lane == 0) {
          atomicAdd(rrow + 2 * DK, dbt);
          atomicAdd(rrow + 2 * DK + 1, dg);
        }
      }
    }
    flush(a, s, x, tok0 + j0, m, (end_read ? 0 : FL_DQ) | FL_DK | FL_SC);
    for (int idx = tid; idx < m * CG; idx += NT) {
      const int t = idx / CG, c = idx % CG;
      a.dv[((int64_t)x.b * a.T + tok0 + j0 + t) * a.lddv + x.hv * DV + x.cg * CG + c] = __float2bfloat16(s.ob[idx]);
    }
  }
}

__global__ void __launch_bounds__(NT) bwd_noisy_kernel(const Args a) {
  extern __shared__ float smem[];
  const int nb = a.L / a.bd;
  Ctx x;
  x.cg = blockIdx.x; x.hv = blockIdx.y;
  const int n = blockIdx.z % nb;
  x.b = blockIdx.z / nb;
  x.tid = threadIdx.x; x.col = x.tid / RP; x.rp = x.tid % RP; x.lane = x.tid & 31; x.par = 0;
  const Stage s = carve(smem, a.bd, true);
  const bool from_clean = noisy_init(a, x.b, n);
  float S0[RPT], dI[RPT];
  const float* ck = state_ptr(a.ckpt, a, x.b, x.hv, n, x.cg);
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    S0[i] = from_clean ? ck[i * NT + x.tid] : 0.f;
    dI[i] = 0.f;
  }
  for (int v = 0; v < a.V; ++v) {
    const int tok0 = (1 + v) * a.L + n * a.bd;
    stage_prepped(a, s, a.qk, a.ab, x.b, x.hv, x.cg, tok0, a.bd, -1, true);
    __syncthreads();
    float dS[RPT];
#pragma unroll
    for (int i = 0; i < RPT; ++i) dS[i] = 0.f;
    bwd_segment(a, s, x, S0, dS, tok0, a.bd, !a.causal_noisy);
#pragma unroll
    for (int i = 0; i < RPT; ++i) dI[i] += dS[i];
    __syncthreads();
  }
  float* di = state_ptr(a.dinit, a, x.b, x.hv, n, x.cg);
#pragma unroll
  for (int i = 0; i < RPT; ++i) di[i * NT + x.tid] = from_clean ? dI[i] : 0.f;
}

__global__ void __launch_bounds__(NT) bwd_clean_kernel(const Args a) {
  extern __shared__ float smem[];
  Ctx x;
  x.cg = blockIdx.x; x.hv = blockIdx.y; x.b = blockIdx.z;
  x.tid = threadIdx.x; x.col = x.tid / RP; x.rp = x.tid % RP; x.lane = x.tid & 31; x.par = 0;
  const Stage s = carve(smem, a.ch, true);
  const int Lc = a.mode ? a.L : a.T;
  const bool end_read = a.mode == 1 && !a.causal_clean;
  float dS[RPT];
#pragma unroll
  for (int i = 0; i < RPT; ++i) dS[i] = 0.f;
  for (int c = a.nch - 1; c >= 0; --c) {
    const int p0 = c * a.ch, n = min(a.ch, Lc - p0);
    float Sst[RPT];
    const float* ck = state_ptr(a.ckpt, a, x.b, x.hv, c, x.cg);
#pragma unroll
    for (int i = 0; i < RPT; ++i) Sst[i] = ck[i * NT + x.tid];
    stage_prepped(a, s, a.qk, a.ab, x.b, x.hv, x.cg, p0, n, p0, true);
    __syncthreads();
    bwd_segment(a, s, x, Sst, dS, p0, n, end_read);
    if (a.mode == 1) {
      const float* di = state_ptr(a.dinit, a, x.b, x.hv, c, x.cg);
#pragma unroll
      for (int i = 0; i < RPT; ++i) dS[i] += di[i * NT + x.tid];
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------------------------
// q/k L2-norm backward (summing the value heads that share a key head) and gate backward
// ---------------------------------------------------------------------------------------------
__global__ void post_bwd_kernel(const Args a, bf16* dmixed, int64_t lddm, bf16* dga, bf16* dgb_out, int64_t lddg,
                                float* dA_log, float* ddt_bias) {
  const int64_t row = blockIdx.x;                   // token b*T + t
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const int rep = a.Hv / a.Hk;
  const bf16* src = a.mixed + row * a.ldm;
  for (int w = warp; w < 2 * a.Hk; w += nw) {
    const int hk = w >> 1, isk = w & 1;
    float xv[4], g[4] = {0.f, 0.f, 0.f, 0.f};
    const bf16* xp = src + isk * a.Hk * DK + hk * DK + lane * 4;
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      xv[e] = __bfloat162float(xp[e]);
      ss += xv[e] * xv[e];
    }
    for (int r = 0; r < rep; ++r)
      for (int c = 0; c < NCG; ++c) {
        const float4 d = *reinterpret_cast<const float4*>(
            a.dpart + ((row * a.Hv + hk * rep + r) * NCG + c) * RED + isk * DK + lane * 4);
        g[0] += d.x; g[1] += d.y; g[2] += d.z; g[3] += d.w;
      }
    ss = warp_sum(ss);
    const float rn = rsqrtf(ss + 1e-6f);
    const float sc = isk ? 1.f : a.scale;
    float dot = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      g[e] *= sc;
      dot += xv[e] * rn * g[e];
    }
    dot = warp_sum(dot);
    bf16* dp = dmixed + row * lddm + isk * a.Hk * DK + hk * DK + lane * 4;
#pragma unroll
    for (int e = 0; e < 4; ++e) dp[e] = __float2bfloat16(rn * (g[e] - xv[e] * rn * dot));
  }
  for (int h = threadIdx.x; h < a.Hv; h += blockDim.x) {
    float dg = 0.f, dbeta = 0.f;
    for (int c = 0; c < NCG; ++c) {
      const float* pr = a.dpart + ((row * a.Hv + h) * NCG + c) * RED + 2 * DK;
      dbeta += pr[0];
      dg += pr[1];
    }
    const float xa = __bfloat162float(a.ga[row * a.ldg + h]) + a.dt_bias[h];
    const float bv = __bfloat162float(a.gb[row * a.ldg + h]);
    const float beta = 1.f / (1.f + expf(-bv));
    const float eA = expf(a.A_log[h]);
    const float sp = softplus_f(xa);
    const float sig = xa > 20.f ? 1.f : 1.f / (1.f + expf(-xa));
    const float da = dg * (-eA) * sig;
    dga[row * lddg + h] = __float2bfloat16(da);
    dgb_out[row * lddg + h] = __float2bfloat16(dbeta * beta * (1.f - beta));
    atomicAdd(dA_log + h, dg * (-eA * sp));
    atomicAdd(ddt_bias + h, da);
  }
}

// ---------------------------------------------------------------------------------------------
// short conv (depthwise, K taps, SiLU), causal or two-stream
// ---------------------------------------------------------------------------------------------
struct ConvArgs {
  int B, T, C, K;
  int mode, L, V, bd;
  const uint8_t* doc;   // [B, Lc]
  const bf16* x; int64_t ldx;
  const bf16* w;        // [C, K]
  bf16* y; int64_t ldy;
};

// Row-relative source token of tap `shift` (reads x[t - shift] in its stream) or -1 (zero pad).
__device__ __forceinline__ int conv_src(const ConvArgs& a, int b, int t, int shift) {
  int stream = 0, p = t;
  if (a.mode) { stream = t / a.L; p = t - stream * a.L; }
  if (p < shift) return -1;
  const int Lc = a.mode ? a.L : a.T;
  if (a.doc != nullptr) {
    const uint8_t* d = a.doc + (int64_t)b * Lc;
    for (int s = 0; s < shift; ++s)
      if (d[p - s]) return -1;    // a document starts inside (p - shift, p]
  }
  if (stream == 0) return t - shift;
  return (p % a.bd) >= shift ? t - shift : p - shift;   // in-block taps: noisy; earlier: clean
}

// The conv kernels give each thread 8 channels of a run of CONV_RUN consecutive tokens of one
// batch row: the 4 x 8 weights stay in registers and the previous rows of the same stream ride in a
// register ring, so a token costs one 16-byte load of x (a tap that reads another stream -- the
// clean prefix of a noisy block -- or a row before the run is loaded on its own).
constexpr int CONV_RUN = 16;

template <int K>
__device__ __forceinline__ void load_w8(const ConvArgs& a, int c8, float (&w)[4][8]) {
#pragma unroll
  for (int e = 0; e < 8; ++e)
#pragma unroll
    for (int j = 0; j < 4; ++j) w[j][e] = j < K ? __bfloat162float(a.w[(c8 + e) * K + j]) : 0.f;
}

__device__ __forceinline__ void zero8(float (&v)[8]) {
#pragma unroll
  for (int e = 0; e < 8; ++e) v[e] = 0.f;
}

// SiLU and the logistic function from the fast exp / divide intrinsics; the exponent is clamped so the
// divisor stays finite (below 2^126, where the fast divide is exact enough for bf16 results).
__device__ __forceinline__ float sigmoid_fast(float x) { return __fdividef(1.f, 1.f + __expf(fminf(-x, 80.f))); }
__device__ __forceinline__ float silu_fast(float x) { return __fdividef(x, 1.f + __expf(fminf(-x, 80.f))); }

// x rows feeding output t: xs[j] for tap j (shift K - 1 - j); ring[i] holds x[t - 1 - i] of the same
// stream when t - 1 - i >= t0 (the run start).
template <int K>
__device__ __forceinline__ void conv_taps(const ConvArgs& a, int b, int t, int t0, int c8, const float (&cur)[8],
                                          const float (&ring)[3][8], float (&xs)[4][8]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int shift = K - 1 - j;
    if (j >= K) { zero8(xs[j]); continue; }
    if (shift == 0) {
#pragma unroll
      for (int e = 0; e < 8; ++e) xs[j][e] = cur[e];
      continue;
    }
    const int src = conv_src(a, b, t, shift);
    if (src < 0) {
      zero8(xs[j]);
    } else if (src == t - shift && src >= t0) {
#pragma unroll
      for (int e = 0; e < 8; ++e) xs[j][e] = ring[shift - 1][e];
    } else {
      load8(a.x + ((int64_t)b * a.T + src) * a.ldx + c8, xs[j]);
    }
  }
}

__device__ __forceinline__ void ring_push(float (&ring)[3][8], const float (&cur)[8]) {
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    ring[2][e] = ring[1][e];
    ring[1][e] = ring[0][e];
    ring[0][e] = cur[e];
  }
}

template <int K>
__global__ void conv_fwd_kernel(const ConvArgs a) {
  const int cpr = a.C / 8;
  const int rpr = (a.T + CONV_RUN - 1) / CONV_RUN;
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (gid >= (int64_t)a.B * rpr * cpr) return;
  const int c8 = (int)(gid % cpr) * 8;
  const int64_t run = gid / cpr;
  const int b = (int)(run / rpr), t0 = (int)(run % rpr) * CONV_RUN, t1 = min(t0 + CONV_RUN, a.T);
  float w[4][8], ring[3][8], cur[8], nxt[8], xs[4][8];
  load_w8<K>(a, c8, w);
  load8(a.x + ((int64_t)b * a.T + t0) * a.ldx + c8, nxt);
  for (int t = t0; t < t1; ++t) {
#pragma unroll
    for (int e = 0; e < 8; ++e) cur[e] = nxt[e];
    // the next row's load is in flight during this row's taps and math
    if (t + 1 < t1) load8(a.x + ((int64_t)b * a.T + t + 1) * a.ldx + c8, nxt);
    conv_taps<K>(a, b, t, t0, c8, cur, ring, xs);
    float out[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float acc = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) acc = fmaf(w[j][e], xs[j][e], acc);
      out[e] = silu_fast(acc);
    }
    store8(a.y + ((int64_t)b * a.T + t) * a.ldy + c8, out);
    ring_push(ring, cur);
  }
}

// dpre = dy * silu'(pre) (fp32), and dw[c, j] += sum_t dpre * x[src] (run partials, one atomic per
// weight per run).
template <int K>
__global__ void conv_bwd_pre_kernel(const ConvArgs a, const bf16* dy, int64_t lddy, float* dpre, float* dw, int) {
  const int cpr = a.C / 8;
  const int rpr = (a.T + CONV_RUN - 1) / CONV_RUN;
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (gid >= (int64_t)a.B * rpr * cpr) return;
  const int c8 = (int)(gid % cpr) * 8;
  const int64_t run = gid / cpr;
  const int b = (int)(run / rpr), t0 = (int)(run % rpr) * CONV_RUN, t1 = min(t0 + CONV_RUN, a.T);
  float w[4][8], ring[3][8], cur[8], xs[4][8], wacc[4][8], nx[8], ndy[8];
  load_w8<K>(a, c8, w);
#pragma unroll
  for (int j = 0; j < 4; ++j) zero8(wacc[j]);
  load8(a.x + ((int64_t)b * a.T + t0) * a.ldx + c8, nx);
  load8(dy + ((int64_t)b * a.T + t0) * lddy + c8, ndy);
  for (int t = t0; t < t1; ++t) {
    const int64_t row = (int64_t)b * a.T + t;
    float dyv[8], g[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      cur[e] = nx[e];
      dyv[e] = ndy[e];
    }
    // the next row's x and dy loads are in flight during this row's taps and math
    if (t + 1 < t1) {
      load8(a.x + (row + 1) * a.ldx + c8, nx);
      load8(dy + (row + 1) * lddy + c8, ndy);
    }
    conv_taps<K>(a, b, t, t0, c8, cur, ring, xs);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float pre = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) pre = fmaf(w[j][e], xs[j][e], pre);
      const float sg = sigmoid_fast(pre);
      g[e] = dyv[e] * sg * (1.f + pre * (1.f - sg));
    }
    float4* dp = reinterpret_cast<float4*>(dpre + row * a.C + c8);
    dp[0] = make_float4(g[0], g[1], g[2], g[3]);
    dp[1] = make_float4(g[4], g[5], g[6], g[7]);
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int e = 0; e < 8; ++e) wacc[j][e] = fmaf(g[e], xs[j][e], wacc[j][e]);
    ring_push(ring, cur);
  }
#pragma unroll
  for (int e = 0; e < 8; ++e)
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (j < K) atomicAdd(dw + (c8 + e) * K + j, wacc[j][e]);
}

__device__ __forceinline__ void load8f(const float* p, float (&v)[8]) {
  const float4 u0 = reinterpret_cast<const float4*>(p)[0], u1 = reinterpret_cast<const float4*>(p)[1];
  v[0] = u0.x; v[1] = u0.y; v[2] = u0.z; v[3] = u0.w; v[4] = u1.x; v[5] = u1.y; v[6] = u1.z; v[7] = u1.w;
}

// dx[s] = sum over outputs t whose tap `shift` reads s of w[c, K-1-shift] * dpre[t].  Same-stream
// outputs s .. s+3 come from a look-ahead ring of dpre rows; a clean row also feeds the first
// in-block taps of every view's noisy block (looked up on their own).
template <int K>
__global__ void conv_bwd_dx_kernel(const ConvArgs a, const float* dpre, bf16* dx, int64_t lddx) {
  const int cpr = a.C / 8;
  const int rpr = (a.T + CONV_RUN - 1) / CONV_RUN;
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (gid >= (int64_t)a.B * rpr * cpr) return;
  const int c8 = (int)(gid % cpr) * 8;
  const int64_t run = gid / cpr;
  const int b = (int)(run / rpr), s0 = (int)(run % rpr) * CONV_RUN, s1 = min(s0 + CONV_RUN, a.T);
  float w[4][8], ahead[4][8];
  load_w8<K>(a, c8, w);
  const float* base = dpre + (int64_t)b * a.T * a.C + c8;
  // ahead[i] = dpre[s + i] (rows past T read as zero)
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    if (s0 + i < a.T) load8f(base + (int64_t)(s0 + i) * a.C, ahead[i]);
    else zero8(ahead[i]);
  }
  for (int s = s0; s < s1; ++s) {
    if (s + 3 < a.T) load8f(base + (int64_t)(s + 3) * a.C, ahead[3]);
    else zero8(ahead[3]);
    float acc[8];
    zero8(acc);
    const int sstream = a.mode ? s / a.L : 0;
    const int lim = a.mode ? (sstream + 1) * a.L : a.T;
#pragma unroll
    for (int shift = 0; shift < 4; ++shift) {
      if (shift >= K) continue;
      const int t = s + shift;
      if (t < lim && conv_src(a, b, t, shift) == s) {
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = fmaf(w[K - 1 - shift][e], ahead[shift][e], acc[e]);
      }
      if (a.mode && sstream == 0) {
        for (int v = 1; v <= a.V; ++v) {
          const int tn = v * a.L + s + shift;
          if (s + shift < a.L && conv_src(a, b, tn, shift) == s) {
            float dv8[8];
            load8f(base + (int64_t)tn * a.C, dv8);
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[e] = fmaf(w[K - 1 - shift][e], dv8[e], acc[e]);
          }
        }
      }
    }
    store8(dx + ((int64_t)b * a.T + s) * lddx + c8, acc);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      ahead[0][e] = ahead[1][e];
      ahead[1][e] = ahead[2][e];
      ahead[2][e] = ahead[3][e];
    }
  }
}

// ---------------------------------------------------------------------------------------------
// gated RMSNorm over the head dim:  y = rmsnorm(o) * w * silu(z)   (one warp per token-head)
// ---------------------------------------------------------------------------------------------
__global__ void gnorm_fwd_kernel(const bf16* o, const bf16* z, int64_t ldz, const bf16* w, bf16* y, int64_t rows,
                                 int H, float eps) {
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= rows * H) return;
  const int64_t row = gw / H;
  const int h = (int)(gw % H);
  const bf16* op = o + gw * DV + lane * 4;
  const bf16* zp = z + row * ldz + h * DV + lane * 4;
  float ov[4], ss = 0.f;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    ov[e] = __bfloat162float(op[e]);
    ss += ov[e] * ov[e];
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / DV + eps);
  bf16* yp = y + gw * DV + lane * 4;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float zv = __bfloat162float(zp[e]);
    const float sz = zv / (1.f + expf(-zv));
    yp[e] = __float2bfloat16(ov[e] * r * __bfloat162float(w[lane * 4 + e]) * sz);
  }
}

__global__ void gnorm_bwd_kernel(const bf16* dy, const bf16* o, const bf16* z, int64_t ldz, const bf16* w, bf16* d_o,
                                 bf16* dz, int64_t lddz, float* dw, int64_t rows, int H, float eps) {
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int lane = threadIdx.x & 31;
  float wacc[4] = {0.f, 0.f, 0.f, 0.f};
  float wv[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) wv[e] = __bfloat162float(w[lane * 4 + e]);
  for (int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; gw < rows * H; gw += nwarps) {
    const int64_t row = gw / H;
    const int h = (int)(gw % H);
    float ov[4], zv[4], dyv[4], ss = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      ov[e] = __bfloat162float(o[gw * DV + lane * 4 + e]);
      zv[e] = __bfloat162float(z[row * ldz + h * DV + lane * 4 + e]);
      dyv[e] = __bfloat162float(dy[gw * DV + lane * 4 + e]);
      ss += ov[e] * ov[e];
    }
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / DV + eps);
    float dn[4], dot = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float sg = 1.f / (1.f + expf(-zv[e]));
      const float sz = zv[e] * sg;
      const float nrm = ov[e] * r;
      const float av = nrm * wv[e];
      dz[row * lddz + h * DV + lane * 4 + e] = __float2bfloat16(dyv[e] * av * sg * (1.f + zv[e] * (1.f - sg)));
      const float da = dyv[e] * sz;
      wacc[e] = fmaf(da, nrm, wacc[e]);
      dn[e] = da * wv[e];
      dot += dn[e] * nrm;
    }
    dot = warp_sum(dot) / DV;
#pragma unroll
    for (int e = 0; e < 4; ++e) d_o[gw * DV + lane * 4 + e] = __float2bfloat16(r * (dn[e] - ov[e] * r * dot));
  }
#pragma unroll
  for (int e = 0; e < 4; ++e) atomicAdd(dw + lane * 4 + e, wacc[e]);
}

}  // namespace gdn

// ---------------------------------------------------------------------------------------------
// launchers
// ---------------------------------------------------------------------------------------------
static gdn::Args make_args(const GdnParams& p) {
  gdn::Args a{};
  a.B = p.B; a.T = p.T; a.Hk = p.Hk; a.Hv = p.Hv;
  a.mode = p.mode; a.L = p.L; a.V = p.V; a.bd = p.bd;
  a.causal_clean = p.causal_clean; a.causal_noisy = p.causal_noisy;
  const int Lc = p.mode ? p.L : p.T;
  a.ch = p.mode ? p.bd : 32;
  a.nch = (Lc + a.ch - 1) / a.ch;
  a.doc = p.doc;
  a.mixed = p.mixed; a.ldm = p.ldm;
  a.ga = p.ga; a.gb = p.gb; a.ldg = p.ldg;
  a.A_log = p.A_log; a.dt_bias = p.dt_bias;
  a.scale = p.scale;
  a.ckpt = p.ckpt; a.o = p.o;
  a.d_o = p.d_o; a.dpart = p.dpart; a.dv = p.dv; a.lddv = p.lddv; a.dinit = p.dinit;
  a.final_state = p.final_state;
  a.qk = p.prep;
  a.ab = p.prep != nullptr ? p.prep + (int64_t)p.B * p.T * 2 * p.Hk * gdn::DK : nullptr;
  return a;
}

int64_t gdn_state_floats(const GdnParams& p) {
  const int Lc = p.mode ? p.L : p.T;
  const int ch = p.mode ? p.bd : 32;
  const int nch = (Lc + ch - 1) / ch;
  return (int64_t)p.B * p.Hv * nch * gdn::DK * gdn::DV;
}

int64_t gdn_part_floats(const GdnParams& p) { return (int64_t)p.B * p.T * p.Hv * gdn::NCG * gdn::RED; }

int gdn_fwd(const GdnParams& p, cudaStream_t st) {
  using namespace gdn;
  if (p.dk != DK || p.dvh != DV || p.Hv % p.Hk) return -1;
  if (p.mode && (p.bd % SUB || p.bd > MAXCH || p.L % p.bd)) return -2;
  const Args a = make_args(p);
  static bool init = false;
  if (!init) {
    const int mx = (int)(stage_floats(MAXCH, false) * sizeof(float));
    cudaFuncSetAttribute(fwd_clean_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
    cudaFuncSetAttribute(fwd_noisy_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
    init = true;
  }
  if (p.prep == nullptr) return -4;
  {
    const int64_t rows = (int64_t)a.B * a.T, warps = rows * (2 * a.Hk + 1);
    prep_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, st>>>(a, p.prep, p.prep + rows * 2 * a.Hk * DK,
                                                                       (int)rows);
  }
  const size_t sm_c = stage_floats(a.ch, false) * sizeof(float);
  fwd_clean_kernel<<<dim3(NCG, a.Hv, a.B), NT, sm_c, st>>>(a);
  if (a.mode && a.V > 0) {
    const size_t sm_n = stage_floats(a.bd, false) * sizeof(float);
    fwd_noisy_kernel<<<dim3(NCG, a.Hv, a.B * (a.L / a.bd)), NT, sm_n, st>>>(a);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int gdn_bwd(const GdnParams& p, bf16* dmixed, int64_t lddm, bf16* dga, bf16* dgb, int64_t lddg, float* dA_log,
            float* ddt_bias, cudaStream_t st) {
  using namespace gdn;
  if (p.dk != DK || p.dvh != DV || p.Hv % p.Hk) return -1;
  if (p.mode && (p.bd % SUB || p.bd > MAXCH || p.L % p.bd)) return -2;
  const Args a = make_args(p);
  static bool init = false;
  if (!init) {
    const int mx = (int)(stage_floats(MAXCH, true) * sizeof(float));
    cudaFuncSetAttribute(bwd_clean_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
    cudaFuncSetAttribute(bwd_noisy_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
    init = true;
  }
  if (p.prep == nullptr) return -4;
  {
    const int64_t rows = (int64_t)a.B * a.T, warps = rows * (2 * a.Hk + 1);
    prep_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, st>>>(a, p.prep, p.prep + rows * 2 * a.Hk * DK,
                                                                       (int)rows);
  }
  if (a.mode && a.V > 0) {
    const size_t sm_n = stage_floats(a.bd, true) * sizeof(float);
    bwd_noisy_kernel<<<dim3(NCG, a.Hv, a.B * (a.L / a.bd)), NT, sm_n, st>>>(a);
  }
  const size_t sm_c = stage_floats(a.ch, true) * sizeof(float);
  bwd_clean_kernel<<<dim3(NCG, a.Hv, a.B), NT, sm_c, st>>>(a);
  post_bwd_kernel<<<(unsigned)(a.B * (int64_t)a.T), 256, 0, st>>>(a, dmixed, lddm, dga, dgb, lddg, dA_log, ddt_bias);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int64_t gdn_prep_floats(int rows, int Hk, int Hv) { return (int64_t)rows * (2 * Hk * gdn::DK + 2 * Hv); }

int gdn_canvas(const GdnParams& p, float* prep, const float* ssm, const int* slot, int n_clean, cudaStream_t st) {
  using namespace gdn;
  if (p.dk != DK || p.dvh != DV || p.Hv % p.Hk || p.T > MAXCH) return -1;
  Args a = make_args(p);
  static bool init = false;
  if (!init) {
    const int mx2 = (int)(canvas2_floats(MAXCH) * sizeof(float));
    cudaFuncSetAttribute(canvas2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, mx2);
    cudaFuncSetAttribute(commit2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, mx2);
    init = true;
  }
  const int rows = a.B * a.T;
  float* qk = prep;
  float* ab = prep + (int64_t)rows * 2 * a.Hk * DK;
  const int64_t warps = (int64_t)rows * (2 * a.Hk + 1);
  prep_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, st>>>(a, qk, ab, rows);
  // two column groups per CTA (see canvas2_kernel)
  canvas2_kernel<<<dim3(NCG / 2, a.Hv, a.B), NT, canvas2_floats(a.T) * sizeof(float), st>>>(a, qk, ab, ssm, slot,
                                                                                          n_clean);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int gdn_commit(const GdnParams& p, const float* prep, float* ssm, const int* slot, const int* adv, cudaStream_t st) {
  using namespace gdn;
  if (p.dk != DK || p.dvh != DV || p.Hv % p.Hk || p.T > MAXCH) return -1;
  Args a = make_args(p);
  const int rows = a.B * a.T;
  const float* qk = prep;
  const float* ab = prep + (int64_t)rows * 2 * a.Hk * DK;
  commit2_kernel<<<dim3(NCG / 2, a.Hv, a.B), NT, canvas2_floats(a.T) * sizeof(float), st>>>(a, qk, ab, ssm, slot,
                                                                                          adv);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

static gdn::ConvArgs conv_args(const ConvParams& p) {
  gdn::ConvArgs a{};
  a.B = p.B; a.T = p.T; a.C = p.C; a.K = p.K;
  a.mode = p.mode; a.L = p.L; a.V = p.V; a.bd = p.bd;
  a.doc = p.doc; a.x = p.x; a.ldx = p.ldx; a.w = p.w; a.y = p.y; a.ldy = p.ldy;
  return a;
}

int gdn_conv_fwd(const ConvParams& p, cudaStream_t st) {
  if (p.C % 8 || p.K > 4 || p.K < 1) return -1;
  const gdn::ConvArgs a = conv_args(p);
  const int64_t n = (int64_t)p.B * ((p.T + gdn::CONV_RUN - 1) / gdn::CONV_RUN) * (p.C / 8);
  const unsigned g = (unsigned)((n + 127) / 128);
  switch (p.K) {
    case 1: gdn::conv_fwd_kernel<1><<<g, 128, 0, st>>>(a); break;
    case 2: gdn::conv_fwd_kernel<2><<<g, 128, 0, st>>>(a); break;
    case 3: gdn::conv_fwd_kernel<3><<<g, 128, 0, st>>>(a); break;
    default: gdn::conv_fwd_kernel<4><<<g, 128, 0, st>>>(a); break;
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int gdn_conv_bwd(const ConvParams& p, const bf16* dy, int64_t lddy, float* dpre, bf16* dx, int64_t lddx, float* dw,
                 cudaStream_t st) {
  if (p.C % 8 || p.K > 4 || p.K < 1) return -1;
  const gdn::ConvArgs a = conv_args(p);
  const int64_t n = (int64_t)p.B * ((p.T + gdn::CONV_RUN - 1) / gdn::CONV_RUN) * (p.C / 8);
  const unsigned g = (unsigned)((n + 127) / 128);
#define TRIDA_CONV_BWD(KK)                                                          \
  gdn::conv_bwd_pre_kernel<KK><<<g, 128, 0, st>>>(a, dy, lddy, dpre, dw, 0);       \
  gdn::conv_bwd_dx_kernel<KK><<<g, 128, 0, st>>>(a, dpre, dx, lddx);
  switch (p.K) {
    case 1: TRIDA_CONV_BWD(1) break;
    case 2: TRIDA_CONV_BWD(2) break;
    case 3: TRIDA_CONV_BWD(3) break;
    default: TRIDA_CONV_BWD(4) break;
  }
#undef TRIDA_CONV_BWD
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int gdn_gnorm_fwd(const bf16* o, const bf16* z, int64_t ldz, const bf16* w, bf16* y, int64_t rows, int H, float eps,
                  cudaStream_t st) {
  const int64_t threads = rows * H * 32;
  gdn::gnorm_fwd_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(o, z, ldz, w, y, rows, H, eps);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int gdn_gnorm_bwd(const bf16* dy, const bf16* o, const bf16* z, int64_t ldz, const bf16* w, bf16* d_o, bf16* dz,
                  int64_t lddz, float* dw, int64_t rows, int H, float eps, int sm_count, cudaStream_t st) {
  const int blocks = sm_count * 8;
  gdn::gnorm_bwd_kernel<<<blocks, 256, 0, st>>>(dy, o, z, ldz, w, d_o, dz, lddz, dw, rows, H, eps);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

}  // namespace trida
