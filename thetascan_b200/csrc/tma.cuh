// Tensor Memory Accelerator (TMA) helpers: tiled bulk-tensor loads of bf16
// tiles into shared memory with the 128-byte swizzle, completion through an
// mbarrier's transaction count, and the tcgen05 shared-memory descriptors that
// read such tiles.
//
// A TMA box of 64 bf16 columns (128 bytes) x R rows lands as R rows of 128
// bytes whose 16-byte chunks are permuted by XOR with (row % 8); the box must
// start on a 1024-byte boundary.  The tensor core reads it as
//   K-major  (rows = M or N, the 64 columns = K): SBO = 1024 (8-row groups),
//            a K step of 16 elements advances the start by 32 bytes inside the
//            128-byte row; the next 64 K-columns are the next box;
//   MN-major (rows = K, the 64 columns = M or N): SBO = 1024 (8-row K groups),
//            LBO = the stride between 64-column boxes, a K step of 16 rows
//            advances the start by 16 * 128 = 2048 bytes.
// No load here uses cluster multicast: every source is this GPU's own memory
// and every destination this CTA's shared memory.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace ts {

constexpr uint32_t kSwBox = 16384;   // one 64-column x 128-row bf16 box
constexpr uint32_t kSwRow = 128;     // bytes per swizzled row
constexpr uint32_t kSwGroup = 1024;  // 8 swizzled rows

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Tiled loads of one box at element coordinates (x = innermost, multiple of 8
// for bf16, then y, z, w) into shared memory at `dst`; the bytes are counted
// on `bar`.  Coordinates past the tensor's extent read zeros.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, int x, int y, int z, int w,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar))
      : "memory");
}

// Untiled bulk copy of `bytes` contiguous bytes (multiple of 16; both
// addresses 16-byte aligned) from global memory into shared memory, counted
// on `bar`.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tma_prefetch_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Byte offset of the 16-byte chunk `c8` (columns 8 c8 .. 8 c8 + 7) of row
// `row` inside a 128-byte-swizzled box (1024-byte aligned): the chunk index
// is XORed with the row's position in its 8-row group.
__device__ __forceinline__ uint32_t sw128_offset(int row, int c8) {
  return static_cast<uint32_t>(row) * kSwRow + static_cast<uint32_t>((c8 ^ (row & 7)) * 16);
}

// Shared-memory descriptor of a 128-byte-swizzled operand (layout type 2).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return smem_desc(saddr, lbo, sbo) | (static_cast<uint64_t>(2) << 61);
}

// In-register transpose of an 8 x 8 block held by 8 consecutive lanes (lane
// l of the group holds row l in x[0..7]); afterwards lane l holds column l.
// Three butterfly rounds: positions whose lane and index differ in bit d
// trade places with the lane d away.  All 32 lanes must call it.
__device__ __forceinline__ void transpose8(float (&x)[8]) {
  const int l = threadIdx.x & 7;
#pragma unroll
  for (int d = 4; d >= 1; d >>= 1) {
    const bool upper = (l & d) != 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if ((i & d) == 0) {
        const float send = upper ? x[i] : x[i | d];
        const float recv = __shfl_xor_sync(0xffffffffu, send, d);
        if (upper) {
          x[i] = recv;
        } else {
          x[i | d] = recv;
        }
      }
    }
  }
}

}  // namespace ts
