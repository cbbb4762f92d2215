// Layout/dtype dispatch for the sm_100a GEMM instantiations.
#include "gemm_sm100.cuh"
namespace trida {
int gemm_tn_bf16(const GemmArgs&, int, int, cudaStream_t);
int gemm_tn_f32(const GemmArgs&, int, int, cudaStream_t);
int gemm_tt_bf16(const GemmArgs&, int, int, cudaStream_t);
int gemm_nt_f32(const GemmArgs&, int, int, cudaStream_t);
int gemm_nt_bf16(const GemmArgs&, int, int, cudaStream_t);

int gemm_bf16(GemmLayout layout, bool d_fp32, const GemmArgs& a, int tile, int sm_count,
              cudaStream_t stream) {
  switch (layout) {
    case GemmLayout::TN:
      return d_fp32 ? gemm_tn_f32(a, tile, sm_count, stream) : gemm_tn_bf16(a, tile, sm_count, stream);
    case GemmLayout::TT:
      return d_fp32 ? -10 : gemm_tt_bf16(a, tile, sm_count, stream);
    case GemmLayout::NT:
      return d_fp32 ? gemm_nt_f32(a, tile, sm_count, stream) : gemm_nt_bf16(a, tile, sm_count, stream);
  }
  return -11;
}
}  // namespace trida
