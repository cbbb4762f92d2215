// bf16 tensor-core GEMM for sm_100a built from CUTLASS/CuTe sm100 collectives.
//
// The mainloop is a warp-specialised TMA -> smem -> tcgen05.mma pipeline with the accumulator in
// TMEM; the epilogue reads TMEM back with tcgen05.ld and stores with TMA.  Only *static* cluster
// shapes (1,1,1) for the 1-SM MMA and (2,1,1) for the 2-SM (cta_group::2) MMA are instantiated:
// with those shapes every TMA load is a plain per-CTA load (no cluster multicast), which keeps the
// kernels legal for operands that live in memory shared with other GPUs.
//
// Row-major torch tensors map to CUTLASS layouts as follows (D is always row-major):
//   fwd    Y[M,N]  = X[M,K] . W[N,K]^T   A=X RowMajor,     B=W ColumnMajor ("TN")
//   dgrad  dX[M,K] = dY[M,N] . W[N,K]    A=dY RowMajor,    B=W RowMajor    ("TT")
//   wgrad  dW[N,K] = dY[M,N]^T . X[M,K]  A=dY ColumnMajor, B=X RowMajor    ("NT")
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

// Returns 0 on success, a negative CUTLASS status code otherwise.  `d_fp32` selects an fp32 D/C
// (weight-gradient accumulation) instead of bf16.  `tile` = 0 picks a tile config by heuristic.
int gemm_bf16(GemmLayout layout, bool d_fp32, const GemmArgs& a, int tile, int sm_count,
              cudaStream_t stream);

}  // namespace trida
