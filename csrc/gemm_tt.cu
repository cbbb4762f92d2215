// Input-gradient GEMM instantiations: dX[M,K] = dY[M,N] . W[N,K] (+ beta*C).
#include "gemm_sm100_impl.cuh"
namespace trida {
int gemm_tt_bf16(const GemmArgs& a, int tile, int sm, cudaStream_t s) {
  return gemm_impl::dispatch<cutlass::layout::RowMajor, cutlass::layout::RowMajor,
                             cutlass::bfloat16_t>(a, tile, sm, s);
}
}  // namespace trida
