// Shared pieces of the tcgen05 block-diffusion attention kernels (head_dim 64 / 128 in
// bd_attention_sm100.cu, head_dim 256 in bd_attention_d256.cu): the token-metadata codes and the
// mask rule of the tile classification, the exp2 and barrier helpers, TMA tensor stores and
// reductions, and the host-side tensor-map builders.
#pragma once

#include <cudaTypedefs.h>

#include "sm100_common.cuh"

namespace trida {
namespace attn100 {

using namespace sm100;

constexpr int SEG_PAD = 0, SEG_SHARED = 1, SEG_XT = 2, SEG_X0 = 3;
constexpr int FLAG_X0_TOKEN_CAUSAL = 1, FLAG_WITHIN_BLOCK_CAUSAL = 2;
constexpr int CLS_FULL = 1;

// Lazy O rescaling: the running max is only moved (and O rescaled in TMEM) when a tile's max
// exceeds it by more than 2^16; until then P = exp2(s - m) <= 65536, far inside bf16/fp32 range,
// and the fp32 accumulators stay exact to their usual rounding.
constexpr float RESCALE_THRESHOLD = 16.0f;   // log2 units

// Branch-free statement of the rule (pure predicate logic: no divergent early returns inside warps).
__device__ __forceinline__ bool allowed(const int4 q, const int4 k, bool same_index, int flags) {
  const int sq = q.w & 0xff, sk = k.w & 0xff;
  const int vq = q.w >> 8, vk = k.w >> 8;
  const bool le = k.x <= q.x;
  const bool to_shared = (sk == SEG_SHARED) & le;
  const bool xt_diag = (sq == SEG_XT) & (sk == SEG_XT) & (q.y == k.y) & (vq == vk) &
                       (((flags & FLAG_WITHIN_BLOCK_CAUSAL) == 0) | le);
  const bool xt_off = (sq == SEG_XT) & (sk == SEG_X0) & (k.y < q.y);
  const bool x0c = (sq == SEG_X0) & (sk == SEG_X0) & (((flags & FLAG_X0_TOKEN_CAUSAL) != 0) ? le : (k.y <= q.y));
  return same_index | ((sk != SEG_PAD) & (q.z == k.z) & (to_shared | xt_diag | xt_off | x0c));
}

// Hardware base-2 exponential (MUFU.EX2 via the PTX ex2.approx instruction); exp2(-inf) = 0.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void named_sync(int id, int n) { asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(n) : "memory"); }

// TMA tensor store of one staged [128 rows][64 bf16] swizzled sub-tile (rows past T are clipped).
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* src, int c0, int c1, int c2, int c3) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];\n" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_addr(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
               : "memory");
}

// TMA tensor reduction: global tile += shared tile (fp32 add), tracked by a bulk group.  The start
// coordinates are never negative (rows past T are clipped by the tensor map bounds).
__device__ __forceinline__ void tma_reduce_add_4d(const CUtensorMap* map, const void* src, int c0, int c1, int c2,
                                                  int c3) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.4d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3, %4, %5}], [%1];\n" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_addr(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;\n" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory"); }

__device__ __forceinline__ void named_bar_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(n) : "memory");
}

// ---- host: tensor maps -------------------------------------------------------------------------
inline PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

// [B, T, H, D] bf16 with element strides (tok, batch); box = 64 x 1 head x 128 tokens x 1.
inline bool make_map(CUtensorMap* m, const void* base, int B, int T, int H, int D, int64_t tok, int64_t bstride) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)T, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)D * 2, (cuuint64_t)tok * 2, (cuuint64_t)bstride * 2};
  cuuint32_t box[4] = {64, 1, 128, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// fp32 [B, T, H, D] contiguous accumulator; box = 32 floats x 1 head x 128 tokens x 1, 128B swizzle.
inline bool make_map_f32(CUtensorMap* m, const void* base, int B, int T, int H, int D) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)T, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)D * 4, (cuuint64_t)H * D * 4, (cuuint64_t)T * H * D * 4};
  cuuint32_t box[4] = {32, 1, 128, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace attn100
}  // namespace trida
