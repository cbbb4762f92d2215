// Template body of the CUTLASS-built sm_100a GEMM; included by one .cu file per layout so the
// (slow) template instantiations compile in parallel.
#pragma once

#include "gemm_sm100.cuh"

#include "cutlass/cutlass.h"
#include "cute/tensor.hpp"
#include "cutlass/numeric_types.h"
#include "cutlass/gemm/dispatch_policy.hpp"
#include "cutlass/gemm/collective/collective_builder.hpp"
#include "cutlass/epilogue/collective/collective_builder.hpp"
#include "cutlass/gemm/device/gemm_universal_adapter.h"
#include "cutlass/gemm/kernel/gemm_universal.hpp"
#include "cutlass/kernel_hardware_info.h"

namespace trida {
namespace gemm_impl {

using namespace cute;

template <class LayoutA, class LayoutB, class ElementD, class MmaTile, class Cluster, bool TwoSm>
struct GemmConfig {
  using ElementA = cutlass::bfloat16_t;
  using ElementB = cutlass::bfloat16_t;
  using ElementC = ElementD;
  using LayoutC = cutlass::layout::RowMajor;
  using ElementAcc = float;
  static constexpr int AlignA = 8;
  static constexpr int AlignB = 8;
  static constexpr int AlignC = 128 / cutlass::sizeof_bits<ElementC>::value;

  using EpiSchedule = cute::conditional_t<TwoSm, cutlass::epilogue::TmaWarpSpecialized2Sm,
                                          cutlass::epilogue::TmaWarpSpecialized1Sm>;
  using MainSchedule = cute::conditional_t<TwoSm, cutlass::gemm::KernelTmaWarpSpecialized2SmSm100,
                                           cutlass::gemm::KernelTmaWarpSpecialized1SmSm100>;

  using CollectiveEpilogue = typename cutlass::epilogue::collective::CollectiveBuilder<
      cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp, MmaTile, Cluster,
      cutlass::epilogue::collective::EpilogueTileAuto, ElementAcc, float,
      ElementC, LayoutC, AlignC, ElementD, LayoutC, AlignC, EpiSchedule>::CollectiveOp;

  using CollectiveMainloop = typename cutlass::gemm::collective::CollectiveBuilder<
      cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp, ElementA, LayoutA, AlignA, ElementB,
      LayoutB, AlignB, ElementAcc, MmaTile, Cluster,
      cutlass::gemm::collective::StageCountAutoCarveout<static_cast<int>(
          sizeof(typename CollectiveEpilogue::SharedStorage))>,
      MainSchedule>::CollectiveOp;

  using Kernel = cutlass::gemm::kernel::GemmUniversal<Shape<int, int, int, int>, CollectiveMainloop,
                                                      CollectiveEpilogue, void>;
  using Gemm = cutlass::gemm::device::GemmUniversalAdapter<Kernel>;
};

// Leading-dimension-aware strides (CUTLASS's packed helpers assume contiguous operands).
template <class Stride, bool RowMajorLike>
Stride make_stride_ld(int64_t ld, int64_t batch_stride) {
  Stride s{};
  if constexpr (RowMajorLike) {
    cute::get<0>(s) = ld;      // (rows, cols:1, batch)
  } else {
    cute::get<1>(s) = ld;      // (rows:1, cols, batch)
  }
  cute::get<2>(s) = batch_stride;
  return s;
}

template <class Cfg>
int run(const GemmArgs& a, int sm_count, cudaStream_t stream) {
  using Gemm = typename Cfg::Gemm;
  using StrideA = typename Gemm::GemmKernel::StrideA;
  using StrideB = typename Gemm::GemmKernel::StrideB;
  using StrideC = typename Gemm::GemmKernel::StrideC;
  using StrideD = typename Gemm::GemmKernel::StrideD;
  using ElementD = typename Cfg::ElementC;

  // StrideA is (M,K,L): K-major (RowMajor A) => (lda, 1, L); M-major => (1, lda, L).
  constexpr bool a_kmajor = cute::is_same_v<decltype(cute::get<1>(StrideA{})), cute::Int<1>>;
  // StrideB is (N,K,L): K-major (ColumnMajor B) => (ldb, 1, L); N-major (RowMajor B) => (1, ldb, L).
  constexpr bool b_kmajor = cute::is_same_v<decltype(cute::get<1>(StrideB{})), cute::Int<1>>;

  StrideA sA = make_stride_ld<StrideA, a_kmajor>(a.lda, a.strideA_batch);
  StrideB sB = make_stride_ld<StrideB, b_kmajor>(a.ldb, a.strideB_batch);
  StrideC sC = make_stride_ld<StrideC, true>(a.ldc, a.strideC_batch);
  StrideD sD = make_stride_ld<StrideD, true>(a.ldd, a.strideD_batch);

  cutlass::KernelHardwareInfo hw;
  hw.device_id = 0;
  hw.sm_count = sm_count;

  typename Gemm::Arguments args{
      cutlass::gemm::GemmUniversalMode::kGemm,
      {a.M, a.N, a.K, a.batch},
      {reinterpret_cast<const cutlass::bfloat16_t*>(a.A), sA,
       reinterpret_cast<const cutlass::bfloat16_t*>(a.B), sB},
      {{a.alpha, a.beta},
       reinterpret_cast<const ElementD*>(a.C ? a.C : a.D), sC,
       reinterpret_cast<ElementD*>(a.D), sD},
      hw};

  Gemm gemm;
  if (gemm.can_implement(args) != cutlass::Status::kSuccess) return -1;
  if (Gemm::get_workspace_size(args) != 0) return -2;   // configs used here need none
  if (gemm.initialize(args, nullptr, stream) != cutlass::Status::kSuccess) return -3;
  if (gemm.run(stream) != cutlass::Status::kSuccess) return -4;
  return 0;
}

// Tile menu: 0 = 2-SM 256x256, 1 = 2-SM 256x128, 2 = 1-SM 128x128 (small problems).
template <class LayoutA, class LayoutB, class ElementD>
int dispatch(const GemmArgs& a, int tile, int sm_count, cudaStream_t stream) {
  if (tile <= 0) {
    const int64_t tiles_big = ((int64_t)(a.M + 255) / 256) * ((a.N + 255) / 256) * a.batch;
    const int64_t tiles_mid = ((int64_t)(a.M + 255) / 256) * ((a.N + 127) / 128) * a.batch;
    if (tiles_big >= sm_count / 2) tile = 1;
    else if (tiles_mid >= sm_count / 4) tile = 2;
    else tile = 3;
  }
  switch (tile) {
    case 1:
      return run<GemmConfig<LayoutA, LayoutB, ElementD, Shape<_256, _256, _64>, Shape<_2, _1, _1>,
                            true>>(a, sm_count, stream);
    case 2:
      return run<GemmConfig<LayoutA, LayoutB, ElementD, Shape<_256, _128, _64>, Shape<_2, _1, _1>,
                            true>>(a, sm_count, stream);
    default:
      return run<GemmConfig<LayoutA, LayoutB, ElementD, Shape<_128, _128, _64>, Shape<_1, _1, _1>,
                            false>>(a, sm_count, stream);
  }
}

}  // namespace gemm_impl
}  // namespace trida
