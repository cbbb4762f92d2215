// Forward-projection GEMM instantiations: Y[M,N] = X[M,K] . W[N,K]^T (+ beta*C).
#include "gemm_sm100_impl.cuh"
namespace trida {
int gemm_tn_bf16(const GemmArgs& a, int tile, int sm, cudaStream_t s) {
  return gemm_impl::dispatch<cutlass::layout::RowMajor, cutlass::layout::ColumnMajor,
                             cutlass::bfloat16_t>(a, tile, sm, s);
}
int gemm_tn_f32(const GemmArgs& a, int tile, int sm, cudaStream_t s) {
  return gemm_impl::dispatch<cutlass::layout::RowMajor, cutlass::layout::ColumnMajor, float>(
      a, tile, sm, s);
}
}  // namespace trida
