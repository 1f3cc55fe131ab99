// Self-test of the tensor-core building blocks: one 128 x N tile product
// D = A . B computed with tcgen05.mma from shared-memory core-matrix tiles,
// with either operand staged K-major or MN-major.  The host compares the
// result with a plain matrix product; a mismatch means a descriptor or tile
// layout error, caught before any real kernel is trusted.
#include "common.cuh"
#include "capi_internal.h"

namespace ts {

__global__ void __launch_bounds__(128) selftest_mma_kernel(const __nv_bfloat16* __restrict__ A,
                                                                const __nv_bfloat16* __restrict__ B,
                                                                float* __restrict__ D, int N, int K,
                                                                int a_mn, int b_mn) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint64_t bar;
  __shared__ uint32_t tmem_base;

  const int tid = threadIdx.x;
  Tile ta = a_mn ? Tile{smem_u32(smem), K, 128} : Tile{smem_u32(smem), 128, K};
  const uint32_t a_bytes = 128u * K * 2u;
  Tile tb = b_mn ? Tile{smem_u32(smem) + a_bytes, K, N} : Tile{smem_u32(smem) + a_bytes, N, K};

  // Stage A (128 x K, row-major in global) and B (K x N, row-major).
  for (int i = tid; i < 128 * K; i += blockDim.x) {
    const int m = i / K, k = i % K;
    const uint32_t off = a_mn ? tile_off(ta, k, m) : tile_off(ta, m, k);
    *reinterpret_cast<__nv_bfloat16*>(smem + (ta.saddr - smem_u32(smem)) + off) = A[i];
  }
  for (int i = tid; i < K * N; i += blockDim.x) {
    const int k = i / N, n = i % N;
    const uint32_t off = b_mn ? tile_off(tb, k, n) : tile_off(tb, n, k);
    *reinterpret_cast<__nv_bfloat16*>(smem + (tb.saddr - smem_u32(smem)) + off) = B[i];
  }
  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  if (tid < 32) tmem_alloc(&tmem_base, 256);
  tiles_ready();

  MmaCtx ctx{&bar, tmem_base, 0u, true};
  const OperandView av = a_mn ? mnmajor(ta) : kmajor(ta);
  const OperandView bv = b_mn ? mnmajor(tb) : kmajor(tb);
  ctx.run([&] { gemm_issue(ctx.tmem, av, bv, N, K, false); });

  const int warp = tid >> 5;
  for (int c = 0; c < N; c += 16) {
    float v[16];
    tmem_ld16(tmem_addr(ctx.tmem, warp * 32, c), v);
#pragma unroll
    for (int e = 0; e < 16; ++e) D[tid * N + c + e] = ctx.ok ? v[e] : __int_as_float(0x7fc00000);
  }
  tc_fence_before();
  __syncthreads();
  if (tid < 32) tmem_dealloc(tmem_base, 256);
}

int selftest_mma(const void* A, const void* B, float* D, int N, int K, int a_mn, int b_mn, cudaStream_t s) {
  if (N < 16 || N > 256 || N % 16 || K < 16 || K > 256 || K % 16) {
    return set_error(TS_ERR_VALUE, "selftest_mma: N and K must be multiples of 16 in [16, 256]");
  }
  const size_t smem = static_cast<size_t>(128 * K + K * N) * 2;
  cudaFuncSetAttribute(selftest_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  selftest_mma_kernel<<<1, 128, smem, s>>>(static_cast<const __nv_bfloat16*>(A),
                                                static_cast<const __nv_bfloat16*>(B), D, N, K, a_mn, b_mn);
  return check_launch("selftest_mma");
}

}  // namespace ts

// ------------------------------------------------------------------ TMA + swizzle

#include "tma.cuh"

namespace ts {

// The same product with both operands brought in by TMA boxes of 64 columns
// with the 128-byte swizzle, read through swizzled descriptors: A as K-major
// (source A [128 x K] row-major) or MN-major (source A^T [K x 128]); B as
// MN-major (source B [K x N]) or K-major (source B^T [N x K]).  N, K in {64, 128}.
__global__ void __launch_bounds__(128) selftest_tma_mma_kernel(const __grid_constant__ CUtensorMap map_a,
                                                                const __grid_constant__ CUtensorMap map_b,
                                                                float* __restrict__ D, int N, int K, int a_mn,
                                                                int b_mn) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t load_bar, bar;
  __shared__ uint32_t tmem_base;
  const int tid = threadIdx.x, warp = tid >> 5;
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t sa = base, sb = base + 128u * K * 2u;
  if (tid == 0) {
    mbar_init(&load_bar, 1);
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(&tmem_base, 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (tid == 0) {
    mbar_expect_tx(&load_bar, static_cast<uint32_t>(128 * K + K * N) * 2u);
    if (a_mn) {
      for (int i = 0; i < 2; ++i) tma_load_2d(sa + i * K * kSwRow, &map_a, i * 64, 0, &load_bar);
    } else {
      for (int i = 0; i < K / 64; ++i) tma_load_2d(sa + i * kSwBox, &map_a, i * 64, 0, &load_bar);
    }
    if (b_mn) {
      for (int i = 0; i < N / 64; ++i) tma_load_2d(sb + i * K * kSwRow, &map_b, i * 64, 0, &load_bar);
    } else {
      for (int i = 0; i < K / 64; ++i) tma_load_2d(sb + i * N * kSwRow, &map_b, i * 64, 0, &load_bar);
    }
  }
  bool ok = mbar_wait(&load_bar, 0, kErrCopyTimeout);
  tc_fence_after();
  if (tid == 0 && ok) {
    const uint32_t id = idesc_bf16(128, N, a_mn != 0, b_mn != 0);
    for (int s = 0; s < K / 16; ++s) {
      const uint64_t ad = a_mn ? smem_desc_sw128(sa + s * 16 * kSwRow, K * kSwRow, kSwGroup)
                               : smem_desc_sw128(sa + (s / 4) * kSwBox + (s % 4) * 32, 0, kSwGroup);
      const uint64_t bd = b_mn ? smem_desc_sw128(sb + s * 16 * kSwRow, K * kSwRow, kSwGroup)
                               : smem_desc_sw128(sb + (s / 4) * N * kSwRow + (s % 4) * 32, 0, kSwGroup);
      mma_bf16(tmem_base, ad, bd, id, s > 0 ? 1u : 0u);
    }
    mma_commit(&bar);
  }
  if (ok) ok = mbar_wait(&bar, 0, kErrMmaTimeout);
  tc_fence_after();
  for (int c = 0; c < N; c += 16) {
    float v[16];
    tmem_ld16(tmem_addr(tmem_base, warp * 32, c), v);
#pragma unroll
    for (int e = 0; e < 16; ++e) D[tid * N + c + e] = ok ? v[e] : __int_as_float(0x7fc00000);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem_base, 256);
}

int selftest_tma_mma(const void* A, const void* B, float* D, int N, int K, int a_mn, int b_mn, cudaStream_t s) {
  if ((N != 64 && N != 128) || (K != 64 && K != 128))
    return set_error(TS_ERR_VALUE, "selftest_tma_mma: N and K must be 64 or 128");
  CUtensorMap ma, mb;
  const uint32_t box_a[2] = {64u, static_cast<uint32_t>(a_mn ? K : 128)};
  const uint64_t dims_a[2] = {static_cast<uint64_t>(a_mn ? 128 : K), static_cast<uint64_t>(a_mn ? K : 128)};
  const int64_t stride_a[1] = {a_mn ? 128 : K};
  const uint32_t box_b[2] = {64u, static_cast<uint32_t>(b_mn ? K : N)};
  const uint64_t dims_b[2] = {static_cast<uint64_t>(b_mn ? N : K), static_cast<uint64_t>(b_mn ? K : N)};
  const int64_t stride_b[1] = {b_mn ? N : K};
  if (!make_tmap_bf16_sw128(&ma, A, 2, dims_a, stride_a, box_a) ||
      !make_tmap_bf16_sw128(&mb, B, 2, dims_b, stride_b, box_b))
    return set_error(TS_ERR_CUDA, "selftest_tma_mma: tensor map encoding failed");
  // 32 KB of slack after the operands: a descriptor misread stays inside the allocation
  const size_t smem = 1024 + static_cast<size_t>(128 * K + K * N) * 2 + 32768;
  cudaFuncSetAttribute(selftest_tma_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  selftest_tma_mma_kernel<<<1, 128, smem, s>>>(ma, mb, D, N, K, a_mn, b_mn);
  return check_launch("selftest_tma_mma");
}

}  // namespace ts
