// Weight-gradient GEMM instantiations: dW[N,K] = dY[M,N]^T . X[M,K] (+ beta*C), fp32 or bf16 out.
#include "gemm_sm100_impl.cuh"
namespace trida {
int gemm_nt_f32(const GemmArgs& a, int tile, int sm, cudaStream_t s) {
  return gemm_impl::dispatch<cutlass::layout::ColumnMajor, cutlass::layout::RowMajor, float>(
      a, tile, sm, s);
}
int gemm_nt_bf16(const GemmArgs& a, int tile, int sm, cudaStream_t s) {
  return gemm_impl::dispatch<cutlass::layout::ColumnMajor, cutlass::layout::RowMajor,
                             cutlass::bfloat16_t>(a, tile, sm, s);
}
}  // namespace trida
