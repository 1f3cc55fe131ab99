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
