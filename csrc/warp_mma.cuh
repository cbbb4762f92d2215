// Warp-level tensor-core helpers shared by the attention kernels: cp.async, ldmatrix,
// mma.sync m16n8k16 (bf16 in, fp32 accumulate), and the XOR-swizzled [rows][D] bf16 tile layout
// that keeps ldmatrix bank-conflict free.
#pragma once

#include "common.cuh"

namespace trida {
namespace attn {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool pred) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(smem)), "l"(gmem),
               "r"(pred ? 16 : 0));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Swizzled element offset of (row, col) in a [rows][D] bf16 tile: 16-byte chunks XOR (row & 7).
template <int D>
__device__ __forceinline__ int swz(int row, int col) {
  const int chunk = (col >> 3) ^ (row & 7);
  return row * D + (chunk << 3) + (col & 7);
}

// Copy a [ROWS][D] tile (rows r0.. of a strided matrix) into swizzled smem with cp.async.
template <int D, int ROWS, int NT>
__device__ __forceinline__ void load_tile(bf16* s, const bf16* g, int64_t ld, int r0, int T) {
  constexpr int CHUNKS = ROWS * D / 8;
  for (int c = threadIdx.x; c < CHUNKS; c += NT) {
    const int row = c / (D / 8), col = (c % (D / 8)) * 8;
    const int gr = r0 + row;
    const bool ok = gr < T;
    cp_async16(s + swz<D>(row, col), g + (int64_t)(ok ? gr : 0) * ld + col, ok);
  }
}

}  // namespace attn
}  // namespace trida
