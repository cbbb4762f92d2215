// bf16 tensor-core GEMM for sm_100a (hand-written tcgen05 / TMA kernel in gemm_sm100.cu).
//
// Layouts of the row-major torch operands (D is always row-major [M, N]):
//   fwd    Y[M,N]  = X[M,K] . W[N,K]^T   A K-major, B K-major  ("TN")
//   dgrad  dX[M,K] = dY[M,N] . W[N,K]    A K-major, B N-major  ("TT")
//   wgrad  dW[N,K] = dY[M,N]^T . X[M,K]  A M-major, B N-major  ("NT")
#pragma once

#include <cuda_runtime.h>
#include <cstdint>

namespace trida {

enum class GemmLayout : int { TN = 0, TT = 1, NT = 2 };

struct GemmArgs {
  int M, N, K;
  const void* A; int64_t lda;   // leading dimension in elements
  const void* B; int64_t ldb;
  const void* C; int64_t ldc;   // may be null when beta == 0
  void* D;       int64_t ldd;
  float alpha, beta;
  int batch;                    // batched GEMM count (strided); 1 for plain GEMM
  int64_t strideA_batch, strideB_batch, strideC_batch, strideD_batch;
};

// Returns 0 on success, a negative code otherwise.  `d_fp32` selects an fp32 D/C (weight-gradient
// accumulation) instead of bf16.  `tile` is reserved (one tile shape is built).
// `splits` > 1 splits K over that many CTAs per output tile (for skinny GEMMs that would leave SMs
// idle): fp32 partials go to `ws` ([splits, M, N]) and a second kernel reduces them into D.
int gemm_bf16(GemmLayout layout, bool d_fp32, const GemmArgs& a, int tile, int sm_count,
              cudaStream_t stream, int splits = 1, float* ws = nullptr);
// K splits gemm_bf16 should use for this shape (1 = none).
int gemm_splitk(int M, int N, int K, int sm_count);

// Tensor-parallel row-parallel GEMM with the all-reduce fused into the epilogue (TN layout, bf16 D,
// D = alpha * sum over ranks of A_r B_r^T + beta * C).  `recv[r]` / `flags[r]`: rank r's receive
// buffer ([2][world][mcap][N] bf16) and arrival counters ([2][tiles_cap][4] u32, zeroed once), as
// mapped into this process; `ctr` / `done`: this rank's call counter and finished-CTA count.
struct GemmAllreduce {
  int world, rank, tiles_cap;
  int64_t mcap;
  void* const* recv;
  unsigned* const* flags;
  unsigned* ctr;
  unsigned* done;
  // optional split K for skinny products: fp32 workspace of ws_units 128 x 256 tiles and arrival
  // counters [tiles_cap][4] (zeroed once), both in this GPU's memory; null = no split
  float* ws;
  int64_t ws_units;
  unsigned* tile_ctr;
};
int gemm_bf16_allreduce(const GemmArgs& a, const GemmAllreduce& ar, int sm_count, cudaStream_t stream);

// Gate / up projection with SwiGLU in the epilogue (TN, bf16): B = [gate; up] ([2F, K], F a multiple
// of 64), D = gu = alpha * A B^T ([M, 2F]) and act = silu(gu[:, :F]) * gu[:, F:] ([M, F]) from the
// bf16-rounded gu values, in one kernel.  `tile`: 0 picks the tile height, 1 = 128 rows, 2 = 256.
// Greedy tokens of D = A B^T (TN, the LM head) without writing D: the epilogue keeps, per row and
// 256-column tile, the max and its column ([M, gemm_argmax_tiles(N)] in am_val / am_idx), and a
// second kernel reduces the tiles into out[M] (int64; the first column on ties).
int gemm_argmax_tiles(int N);
int gemm_bf16_argmax(const GemmArgs& a, float* am_val, int* am_idx, int64_t* out, int sm_count, cudaStream_t stream);

int gemm_bf16_swiglu(const GemmArgs& a, void* act, int64_t ld_act, int F, int tile, int sm_count,
                     cudaStream_t stream);

// Device int the GEMM's bounded mbarrier waits set (non-zero) on a timeout; null if unallocated.
int* gemm_error_word();

}  // namespace trida
