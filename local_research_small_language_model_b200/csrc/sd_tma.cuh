// TMA tensor maps (host encode) and the tensor-copy / ldmatrix / mma.sync
// wrappers used by the 16-bit decode attention path.
#pragma once

#include <cuda.h>

#include "sd_common.cuh"

namespace sd {

// Encodes a 4-D row map over a [B][H][T][D] tensor of 16-bit elements
// (strides in elements, innermost 1), box = box_rows x D, 128-byte swizzle.
// D * 2 must be 128 (one swizzle atom per row).  Returns SD_OK or an error.
int encode_rows_map(CUtensorMap *map, const void *base, int dtype, int64_t D, int64_t T, int64_t H, int64_t B,
                    int64_t st, int64_t sh, int64_t sb, int box_rows);

// Encodes a 2-D tiled map over a row-major [rows][cols] matrix of 16-bit
// elements (row stride `ld` elements), box = box_rows x 64 columns (128
// bytes, one swizzle atom), 128-byte swizzle; rows past `rows` read as zero.
int encode_matrix_map(CUtensorMap *map, const void *base, int dtype, int64_t rows, int64_t cols, int64_t ld,
                      int box_rows);

// As encode_matrix_map, with a box of box_rows x box_cols (box_cols a
// multiple of 8) and no swizzle: the box lands row-major in shared memory.
int encode_plain_map(CUtensorMap *map, const void *base, int dtype, int64_t rows, int64_t cols, int64_t ld,
                     int box_cols, int box_rows);

__device__ __forceinline__ void tma_load_2d(void *smem_dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------- device side
__device__ __forceinline__ void tma_load_4d(void *smem_dst, const CUtensorMap *map, int x, int y, int z, int w,
                                            uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// D(16x8, fp32) += A(16x16) * B(16x8), 16-bit inputs.
template <typename T> __device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                                               uint32_t b1);
template <> __device__ __forceinline__ void mma16816<__nv_bfloat16>(float (&d)[4], const uint32_t (&a)[4],
                                                                     uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <> __device__ __forceinline__ void mma16816<__half>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                                              uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Packs two floats into a 16-bit pair (lo = first element).
template <typename T> __device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <> __device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&v);
}
template <> __device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&v);
}

// Byte offset of (row, 16-byte chunk) in a tile written by a 128-byte-swizzle
// TMA copy with 128-byte rows (chunk index XOR row mod 8).
__device__ __forceinline__ uint32_t sw128(int row, int chunk) {
  return static_cast<uint32_t>(row * 128 + (((chunk ^ (row & 7)) & 7) << 4));
}

}  // namespace sd
