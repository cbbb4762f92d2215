// Device-side sampler of the self-speculative decode step (sampled requests).
//
// Per request (one warp): the canvas rows' candidate lists (the top KMAX logits per row, sorted,
// from one batched top-k pass over the logits) become truncated distributions -- softmax of
// logits / T over the request's top-k, then the nucleus cut (a candidate is dropped when the mass
// of the candidates before it already exceeds top_p), renormalised -- and then:
//   * a request without drafts (its first canvas) samples rows 0 .. n-1: row 0 is the next token,
//     rows 1 .. n-1 are the drafts, and their distributions are kept as the drafts' q lists;
//   * a request with drafts d_0 .. d_{K-1} verifies them in order (speculative sampling): draft j
//     is kept when u < p_j(d_j) / q_j(d_j); at the first rejection the correction is drawn from
//     the residual max(p_j - q_j, 0) (p_j when the residual is empty); when all K are kept, rows
//     n-1 .. blk-1 are sampled: the bonus token, then new drafts with their q lists.
// Tokens are drawn by inverse CDF over the candidates with uniforms from SplitMix64 (Steele, Lea
// and Flood, "Fast splittable pseudorandom number generators", OOPSLA 2014) of (seed, counter);
// the counter lives on the device per slot and advances with every draw, so a seeded request
// reproduces its samples regardless of batching.  Outputs per request: accepted count, correction
// (or -1), next clean token, the new drafts; q lists are written in place per slot.
#include "common.cuh"
#include "ops.h"

namespace trida {
namespace spec {

constexpr int KMAX = 64;       // candidates per row (two per lane)

struct Args {
  const float* vals;      // [B, blk, kc] candidate logits, sorted descending
  const int64_t* idx;     // [B, blk, kc] candidate token ids
  int kc;                 // candidates per row in vals / idx (<= KMAX)
  const float* temp;      // [B]
  const int* topk;        // [B] (<= kc)
  const float* topp;      // [B]
  const int64_t* seed;    // [B]
  int64_t* counter;       // [slots] draws made so far
  const int* slot;        // [B]
  const int* specs;       // [B, K] drafts (valid when has_specs[b])
  const int* has_specs;   // [B]
  int* q_idx;             // [slots, K, KMAX] draft distributions (token ids, -1 = unused)
  float* q_prob;          // [slots, K, KMAX]
  int* out;               // [B, 3 + K]: accepted, correction, clean, new drafts
  int blk, n, K;
};

__device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

// uniform in [0, 1) from draw number `c` of stream `seed` (24 random bits)
__device__ __forceinline__ float uniform(uint64_t seed, uint64_t c) {
  return (float)(splitmix64(seed ^ splitmix64(c)) >> 40) * (1.0f / 16777216.0f);
}

__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// inclusive prefix sum over the warp's lanes
__device__ __forceinline__ float warp_scan(float v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float t = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += t;
  }
  return v;
}

// Truncated distribution of one row over its candidates: lane l holds candidates l and l + 32.
struct Row {
  float p[2];
  int tok[2];
};

__device__ Row truncated(const Args& a, int b, int row) {
  const int lane = threadIdx.x & 31;
  const int64_t base = ((int64_t)b * a.blk + row) * a.kc;
  const float T = fmaxf(a.temp[b], 1e-6f);
  const int k = min(a.topk[b], a.kc);
  const float mx = a.vals[base] / T;
  Row r;
  float e[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int c = lane + 32 * h;
    r.tok[h] = c < k ? (int)a.idx[base + c] : -1;
    e[h] = c < k ? __expf(a.vals[base + c] / T - mx) : 0.f;
  }
  const float z = warp_sum_f(e[0] + e[1]);
  // nucleus: candidates are sorted, so the mass before candidate c is a prefix sum
  const float c0 = warp_scan(e[0] / z);
  const float tot0 = __shfl_sync(0xffffffffu, c0, 31);
  const float c1 = warp_scan(e[1] / z) + tot0;
  const float tp = a.topp[b];
  const bool keep0 = tp >= 1.f || (c0 - e[0] / z) <= tp;
  const bool keep1 = tp >= 1.f || (c1 - e[1] / z) <= tp;
  e[0] = keep0 ? e[0] : 0.f;
  e[1] = keep1 ? e[1] : 0.f;
  const float z2 = warp_sum_f(e[0] + e[1]);
  r.p[0] = e[0] / z2;
  r.p[1] = e[1] / z2;
  return r;
}

// probability of `tok` under a candidate list held by the warp (0 when absent)
__device__ __forceinline__ float prob_of(const Row& r, int tok) {
  float v = (r.tok[0] == tok ? r.p[0] : 0.f) + (r.tok[1] == tok ? r.p[1] : 0.f);
  return warp_sum_f(v);
}

// inverse-CDF draw from unnormalised weights w (lane l: candidates l, l + 32)
__device__ int draw(const float (&w)[2], const int (&tok)[2], float u) {
  const float s0 = warp_scan(w[0]);
  const float t0 = __shfl_sync(0xffffffffu, s0, 31);
  const float s1 = warp_scan(w[1]) + t0;
  const float tot = __shfl_sync(0xffffffffu, s1, 31);
  const float target = u * tot;
  const unsigned b0 = __ballot_sync(0xffffffffu, w[0] > 0.f && s0 > target);
  const unsigned b1 = __ballot_sync(0xffffffffu, w[1] > 0.f && s1 > target);
  int lane_pick, h;
  if (b0) {
    lane_pick = __ffs(b0) - 1;
    h = 0;
  } else if (b1) {
    lane_pick = __ffs(b1) - 1;
    h = 1;
  } else {   // rounding at the top end: the last candidate with weight
    const unsigned n1 = __ballot_sync(0xffffffffu, w[1] > 0.f), n0 = __ballot_sync(0xffffffffu, w[0] > 0.f);
    h = n1 ? 1 : 0;
    lane_pick = n1 ? 31 - __clz(n1) : (n0 ? 31 - __clz(n0) : 0);
  }
  const int t = h ? tok[1] : tok[0];
  return __shfl_sync(0xffffffffu, t, lane_pick);
}

__device__ __forceinline__ void store_q(const Args& a, int s, int j, const Row& r) {
  const int lane = threadIdx.x & 31;
  const int64_t o = ((int64_t)s * a.K + j) * KMAX;
  a.q_idx[o + lane] = r.p[0] > 0.f ? r.tok[0] : -1;
  a.q_idx[o + lane + 32] = r.p[1] > 0.f ? r.tok[1] : -1;
  a.q_prob[o + lane] = r.p[0];
  a.q_prob[o + lane + 32] = r.p[1];
}

// q_j(tok) from the slot's stored list
__device__ __forceinline__ float q_of(const Args& a, int s, int j, int tok) {
  const int lane = threadIdx.x & 31;
  const int64_t o = ((int64_t)s * a.K + j) * KMAX;
  float v = (a.q_idx[o + lane] == tok ? a.q_prob[o + lane] : 0.f) +
            (a.q_idx[o + lane + 32] == tok ? a.q_prob[o + lane + 32] : 0.f);
  return warp_sum_f(v);
}

__global__ void spec_sample_kernel(const Args a) {
  const int b = blockIdx.x;
  const int lane = threadIdx.x & 31;
  const int s = a.slot[b];
  const uint64_t seed = (uint64_t)a.seed[b];
  uint64_t ctr = (uint64_t)a.counter[s];
  int* out = a.out + (int64_t)b * (3 + a.K);
  const int K = a.K, n = a.n;
  int acc = 0, corr = -1, clean = -1;
  int first_new = 0;          // first canvas row sampled as [clean, drafts...]
  if (a.has_specs[b]) {
    for (acc = 0; acc < K; ++acc) {
      const int d = a.specs[(int64_t)b * K + acc];
      const Row r = truncated(a, b, acc);
      const float p = prob_of(r, d), q = q_of(a, s, acc, d);
      const float u = uniform(seed, ctr++);
      const bool keep = q > 0.f ? (p >= q || u * q < p) : false;
      if (keep) continue;
      // residual max(p - q, 0) over p's candidates (q's mass outside p's support has no residual)
      float w[2];
      for (int h = 0; h < 2; ++h) {
        const int t = r.tok[h];
        float qt = 0.f;
        const int64_t o = ((int64_t)s * K + acc) * KMAX;
        for (int c = 0; c < KMAX; ++c)
          if (a.q_idx[o + c] == t && t >= 0) qt = a.q_prob[o + c];
        w[h] = fmaxf(r.p[h] - qt, 0.f);
      }
      const float tot = warp_sum_f(w[0] + w[1]);
      if (tot <= 0.f) {
        w[0] = r.p[0];
        w[1] = r.p[1];
      }
      corr = draw(w, r.tok, uniform(seed, ctr++));
      break;
    }
    first_new = n - 1;        // all drafts kept: the bonus row, then the new drafts
  }
  if (corr < 0) {
    for (int row = first_new; row < first_new + n; ++row) {
      const Row r = truncated(a, b, row);
      const float w[2] = {r.p[0], r.p[1]};
      const int t = draw(w, r.tok, uniform(seed, ctr++));
      if (row == first_new) {
        clean = t;
      } else {
        if (lane == 0) out[3 + row - first_new - 1] = t;
        store_q(a, s, row - first_new - 1, r);
      }
    }
  }
  if (lane == 0) {
    out[0] = acc;
    out[1] = corr;
    out[2] = clean;
    a.counter[s] = (int64_t)ctr;
  }
}

}  // namespace spec

int spec_sample(const float* vals, const int64_t* idx, int kc, const float* temp, const int* topk, const float* topp,
                const int64_t* seed, int64_t* counter, const int* slot, const int* specs, const int* has_specs,
                int* q_idx, float* q_prob, int* out, int B, int blk, int n, cudaStream_t st) {
  if (kc < 1 || kc > spec::KMAX || n < 1 || blk < n) return -1;
  spec::Args a{vals, idx, kc, temp, topk, topp, seed, counter, slot, specs, has_specs, q_idx, q_prob, out, blk, n,
               n - 1};
  spec::spec_sample_kernel<<<B, 32, 0, st>>>(a);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

}  // namespace trida
