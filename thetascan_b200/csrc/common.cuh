// Shared device helpers for the sm_100a ThetaScan kernels.
//
// Tensor-core work uses the 5th-generation MMA (tcgen05.mma, kind::f16,
// bf16 x bf16 -> f32) with accumulators in Tensor Memory (TMEM).  Operands are
// staged in shared memory as "core-matrix tiles":
//
//   a tile of R rows x C columns of bf16 (R, C multiples of 8) stores element
//   (r, c) at byte  (c/8)*R*16 + (r/8)*128 + (r%8)*16 + (c%8)*2,
//
// i.e. every 8x8 block ("core matrix", 8 rows of 16 contiguous bytes) is one
// 128-byte line, blocks of one 8-column chunk are stacked down the rows, and
// chunks follow each other.  The same bytes can be read by the MMA either as a
// K-major operand (tile rows = M or N, tile columns = K) or as an MN-major
// operand (tile rows = K, tile columns = M or N); only the two strides of the
// shared-memory descriptor differ.  That lets one staged copy of, say, a key
// tile serve both the score product q.k^T and the state update k^T.v.
//
// Every wait on an mbarrier is bounded.  On timeout the kernel records an
// error code in a device flag that the host reads back (ts_b200_device_status)
// and stops issuing work; nothing traps or spins forever.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace ts {

constexpr int kTile = 128;            // tokens per tile (= MMA M)
constexpr int kThreads = 512;         // threads of a tile CTA
constexpr int kParts = kThreads / kTile;  // threads per tile row
constexpr int kChunkStep = 16 * kParts;   // column stride between a thread's 16-column chunks

// Thread <-> (tile row, part).  Warps w, w+4, w+8 and w+12 read the same TMEM
// lane quadrant (w % 4), so threads t + 128 j (j < kParts) own the same
// accumulator row and split its columns into 16-column chunks dealt out in
// turn: part j takes chunks j, j + kParts, ...
__device__ __forceinline__ int my_row() { return threadIdx.x & (kTile - 1); }
__device__ __forceinline__ int my_part() { return threadIdx.x >> 7; }
__device__ __forceinline__ int my_quad() { return (threadIdx.x >> 5) & 3; }

// Error codes written to the device status word.
enum DeviceError : int {
  kErrNone = 0,
  kErrMmaTimeout = 1,
  kErrCopyTimeout = 2,
};

// Device status word (the library is one translation unit; see all.cu).
__device__ int g_device_status = 0;

__device__ __forceinline__ void record_error(int code) {
  atomicCAS(&g_device_status, 0, code);
}

__device__ __forceinline__ bool device_failed() {
  return *(volatile int*)&g_device_status != 0;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------------ mbarrier

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Wait for the phase with the given parity to complete.  Gives up after about
// one second (or 2^24 polls), records `code` and returns false.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = globaltimer_ns();
  for (uint32_t i = 0; i < (1u << 24); ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 255u) {
      if (globaltimer_ns() - start > 1000000000ull) break;
      if (device_failed()) return false;
    }
  }
  record_error(code);
  return false;
}

// ------------------------------------------------------------------ tcgen05

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Make this thread's generic-proxy shared-memory writes visible to the async
// proxy (the tensor core reads operands through it).
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Warp-wide: allocate `ncols` TMEM columns (power of two >= 32); the base
// address is written to *dst.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// Instruction descriptor for kind::f16 with bf16 A/B and an f32 accumulator.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, bool a_mn_major, bool b_mn_major) {
  return (1u << 4)                                  // D format: f32
         | (1u << 7)                                // A format: bf16
         | (1u << 10)                               // B format: bf16
         | (static_cast<uint32_t>(a_mn_major) << 15)
         | (static_cast<uint32_t>(b_mn_major) << 16)
         | (static_cast<uint32_t>(N >> 3) << 17)
         | (static_cast<uint32_t>(M >> 4) << 24);
}

// Shared-memory matrix descriptor, no swizzle (layout type 0), sm_100 version 1.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  return d;
}

__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on `bar` when every MMA previously issued by this thread completes.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// Warp-collective: 16 consecutive 32-bit TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Warp-collective: columns [c_k, c_k + 16) of this lane's row for four
// column offsets c_k = c0 + k * stride, with one wait for all four loads (the
// wait is part of the same asm statement, so no use of the registers can be
// scheduled before it).
__device__ __forceinline__ void tmem_ld16x4(uint32_t taddr, uint32_t stride, float (&v)[4][16]) {
  uint32_t r[64];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%64];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%65];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47}, [%66];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%67];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
        "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
        "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
        "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
        "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr), "r"(taddr + stride), "r"(taddr + 2 * stride), "r"(taddr + 3 * stride)
      : "memory");
#pragma unroll
  for (int k = 0; k < 4; ++k)
#pragma unroll
    for (int i = 0; i < 16; ++i) v[k][i] = __uint_as_float(r[16 * k + i]);
}

// Warp-collective: write 16 consecutive 32-bit TMEM columns of this lane.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15]))
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// TMEM address of (lane, column): lane in bits 31:16, column in 15:0.
__device__ __forceinline__ uint32_t tmem_addr(uint32_t base, int lane, int col) {
  return base + (static_cast<uint32_t>(lane) << 16) + static_cast<uint32_t>(col);
}

// ------------------------------------------------------------------ tiles

struct Tile {
  uint32_t saddr;  // shared-memory byte address (16-byte aligned)
  int rows;        // multiple of 8
  int cols;        // multiple of 8
};

__device__ __forceinline__ uint32_t tile_off(const Tile& t, int r, int c) {
  return static_cast<uint32_t>((c >> 3) * t.rows * 16 + (r >> 3) * 128 + (r & 7) * 16 + (c & 7) * 2);
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}

// 16 bytes = columns c8*8 .. c8*8+7 of row r.
__device__ __forceinline__ void tile_st16(const Tile& t, int r, int c8, uint4 v) {
  st_shared_v4(t.saddr + tile_off(t, r, c8 * 8), v);
}
__device__ __forceinline__ uint4 tile_ld16(const Tile& t, int r, int c8) {
  return ld_shared_v4(t.saddr + tile_off(t, r, c8 * 8));
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ float2 unpack_bf16(uint32_t u) {
  __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162*>(&u);
  return __bfloat1622float2(h);
}
__device__ __forceinline__ uint4 pack8(const float* f) {
  return make_uint4(pack_bf16(f[0], f[1]), pack_bf16(f[2], f[3]), pack_bf16(f[4], f[5]),
                    pack_bf16(f[6], f[7]));
}
__device__ __forceinline__ void unpack8(uint4 u, float* f) {
  float2 a = unpack_bf16(u.x), b = unpack_bf16(u.y), c = unpack_bf16(u.z), d = unpack_bf16(u.w);
  f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y; f[4] = c.x; f[5] = c.y; f[6] = d.x; f[7] = d.y;
}

// Operand views of a tile for the descriptor.  `r0`/`c0` select a sub-block
// (r0 multiple of 8, c0 multiple of 8).
//
// K-major view: MMA rows (M or N) = tile rows, K = tile columns.
//   LBO = stride between 8-column K groups = rows*16, SBO = 128.
// MN-major view: K = tile rows, MMA rows/cols (M or N) = tile columns.
//   SBO = stride between 8-column MN groups = rows*16, LBO = 128.
struct OperandView {
  uint32_t start;
  uint32_t lbo, sbo;
  uint32_t kstep;  // bytes to advance per K step of 16
  bool mn_major;
};

__device__ __forceinline__ OperandView kmajor(const Tile& t, int r0 = 0, int c0 = 0) {
  OperandView v;
  v.start = t.saddr + tile_off(t, r0, c0);
  v.lbo = static_cast<uint32_t>(t.rows * 16);
  v.sbo = 128u;
  v.kstep = static_cast<uint32_t>(2 * t.rows * 16);
  v.mn_major = false;
  return v;
}
__device__ __forceinline__ OperandView mnmajor(const Tile& t, int r0 = 0, int c0 = 0) {
  OperandView v;
  v.start = t.saddr + tile_off(t, r0, c0);
  v.lbo = 128u;
  v.sbo = static_cast<uint32_t>(t.rows * 16);
  v.kstep = 256u;
  v.mn_major = true;
  return v;
}

// D[128 x N] (+)= A[128 x K] . B[K x N]; issue from ONE thread.  K multiple
// of 16, N multiple of 16 in [16, 256].
__device__ __forceinline__ void gemm_issue(uint32_t d_tmem, const OperandView& a, const OperandView& b, int N,
                                           int K, bool accumulate) {
  const uint32_t id = idesc_bf16(128, N, a.mn_major, b.mn_major);
  for (int s = 0; s < K / 16; ++s) {
    const uint64_t ad = smem_desc(a.start + s * a.kstep, a.lbo, a.sbo);
    const uint64_t bd = smem_desc(b.start + s * b.kstep, b.lbo, b.sbo);
    mma_bf16(d_tmem, ad, bd, id, (accumulate || s > 0) ? 1u : 0u);
  }
}

// ------------------------------------------------------------------ loads

__device__ __forceinline__ float bf2f(__nv_bfloat16 x) { return __bfloat162float(x); }

// 16-byte asynchronous global -> shared copy (LDGSTS, L1 bypassed).  Many
// can be in flight per thread; cp_async_wait_all() waits for this thread's.
__device__ __forceinline__ void cp_async16(uint32_t saddr, const void* gptr) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr), "l"(gptr) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}
// Close the current group of this thread's cp.async copies / wait until at
// most the newest `N` committed groups are still in flight.
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait_group() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Cooperative copy of a row-major bf16 matrix (rows_valid x cols_valid,
// leading dimension `ld` elements) into `t`, zero-filling the rest of the
// tile.  Consecutive threads cover 8 rows of one 8-column chunk, so the shared
// stores are conflict-free and each row is read in 64-byte runs.  If
// `unit_col` >= 0, columns [unit_col, unit_col + unit_count) of every valid
// row are set to 1.
// Whole in-range 16-byte chunks are copied with cp.async, so a thread has all
// of its copies in flight at once; the tile is complete after
// cp_async_wait_all() (MmaCtx::run and tiles_ready() do that) and a barrier.
__device__ __forceinline__ void load_tile(const Tile& t, const __nv_bfloat16* __restrict__ src, long ld,
                                          int rows_valid, int cols_valid, int unit_col = -1,
                                          int unit_count = 1) {
  const int chunks = t.cols / 8;
  const int total = t.rows * chunks;
  const bool vec_ok = ((reinterpret_cast<uintptr_t>(src) & 15) == 0) && ((ld & 7) == 0);
  for (int it = threadIdx.x; it < total; it += blockDim.x) {
    const int r8 = it & 7;
    const int rest = it >> 3;
    const int j = rest % chunks;
    const int r = (rest / chunks) * 8 + r8;
    const int c0 = j * 8;
    const bool has_unit = unit_col >= 0 && unit_col < c0 + 8 && unit_col + unit_count > c0;
    if (r < rows_valid && vec_ok && c0 + 8 <= cols_valid && !has_unit) {
      cp_async16(t.saddr + tile_off(t, r, c0), src + r * ld + c0);
      continue;
    }
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < rows_valid) {
      float f[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int c = c0 + e;
        f[e] = (c < cols_valid) ? bf2f(src[r * ld + c]) : 0.f;
      }
      if (has_unit) {
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (c0 + e >= unit_col && c0 + e < unit_col + unit_count) f[e] = 1.f;
      }
      v = pack8(f);
    }
    tile_st16(t, r, j, v);
  }
}

// Cooperative, coalesced copy of a tile back to a row-major bf16 matrix
// (rows_valid x cols_valid, leading dimension `ld`): the inverse of load_tile.
__device__ __forceinline__ void store_tile(const Tile& t, __nv_bfloat16* __restrict__ dst, long ld, int rows_valid,
                                           int cols_valid) {
  const int chunks = t.cols / 8;
  const int total = t.rows * chunks;
  const bool vec_ok = ((reinterpret_cast<uintptr_t>(dst) & 15) == 0) && ((ld & 7) == 0);
  for (int it = threadIdx.x; it < total; it += blockDim.x) {
    const int r8 = it & 7;
    const int rest = it >> 3;
    const int j = rest % chunks;
    const int r = (rest / chunks) * 8 + r8;
    const int c0 = j * 8;
    if (r >= rows_valid || c0 >= cols_valid) continue;
    const uint4 v = tile_ld16(t, r, j);
    if (vec_ok && c0 + 8 <= cols_valid) {
      *reinterpret_cast<uint4*>(dst + r * ld + c0) = v;
    } else {
      float f[8];
      unpack8(v, f);
      #pragma unroll
      for (int e = 0; e < 8; ++e)
        if (c0 + e < cols_valid) dst[r * ld + c0 + e] = __float2bfloat16_rn(f[e]);
    }
  }
}

// Coalesced store of accumulator rows.  The kParts threads of row r own row
// r of a TMEM accumulator (columns [0, ncols) starting at column `tcol` of
// `tbase`); rows [0, rows_valid) and columns [0, width) go to the row-major
// matrix `dst` with leading dimension `ld` (f32 or bf16).  Every kChunkStep
// columns pass through a shared stage of kTile * kChunkStep floats (32 KB),
// XOR-swizzled so that both the row-wise writes and the column-wise reads are
// free of bank conflicts, and leave as whole 32-byte sectors.
// `transform(row, col, value)` may adjust each value; `addend` (same layout as
// dst, f32) is added on the way out.  With tcol_b >= 0 the value is
// A + scale_b * B, B the accumulator at TMEM column tcol_b and scale_b this
// thread's row factor.
constexpr int kStageFloats = kTile * kChunkStep;

__device__ __forceinline__ int stage_idx(int r, int c) { return r * kChunkStep + (c ^ (r & 31)); }

template <class Transform>
__device__ __forceinline__ void store_rows(uint32_t tbase, int tcol, int ncols, int width, int rows_valid, void* dst,
                                           long ld, bool bf16, float* stage, Transform transform,
                                           const float* __restrict__ addend = nullptr, int tcol_b = -1,
                                           float scale_b = 0.f) {
  const int row = my_row(), part = my_part();
  const uint32_t trow = tmem_addr(tbase, my_quad() * 32, tcol);
  const uint32_t trow_b = tmem_addr(tbase, my_quad() * 32, tcol_b < 0 ? 0 : tcol_b);
  for (int c = 0; c < ncols; c += kChunkStep) {
    const int cc = c + 16 * part;
    if (cc < ncols) {
      float v[16];
      tmem_ld16(trow + cc, v);
      if (tcol_b >= 0) {
        // a second accumulator of the same shape, scaled per row (this thread's)
        float w[16];
        tmem_ld16(trow_b + cc, w);
#pragma unroll
        for (int e = 0; e < 16; ++e) v[e] = fmaf(scale_b, w[e], v[e]);
      }
#pragma unroll
      for (int e = 0; e < 16; ++e) stage[stage_idx(row, 16 * part + e)] = transform(row, cc + e, v[e]);
    }
    __syncthreads();
    const int cols = min(kChunkStep, width - c);
    if (cols > 0) {
      // 8 consecutive columns per thread: one 16-byte store (bf16) or two (f32)
      // where the row segment is whole and aligned, element stores otherwise.
      constexpr int kGroups = kChunkStep / 8;
      for (int i = threadIdx.x; i < rows_valid * kGroups; i += blockDim.x) {
        const int r = i / kGroups, e0 = (i % kGroups) * 8;
        if (e0 >= cols) continue;
        float x[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) x[q] = stage[stage_idx(r, e0 + q)];
        const long off = r * ld + c + e0;
        const bool whole = e0 + 8 <= cols;
        if (addend != nullptr) {
#pragma unroll
          for (int q = 0; q < 8; ++q)
            if (whole || e0 + q < cols) x[q] += addend[off + q];
        }
        if (bf16) {
          __nv_bfloat16* d = reinterpret_cast<__nv_bfloat16*>(dst) + off;
          if (whole && (reinterpret_cast<uintptr_t>(d) & 15) == 0) {
            *reinterpret_cast<uint4*>(d) = pack8(x);
          } else {
            #pragma unroll
            for (int q = 0; q < 8; ++q)
              if (e0 + q < cols) d[q] = __float2bfloat16_rn(x[q]);
          }
        } else {
          float* d = reinterpret_cast<float*>(dst) + off;
          if (whole && (reinterpret_cast<uintptr_t>(d) & 15) == 0) {
            reinterpret_cast<float4*>(d)[0] = make_float4(x[0], x[1], x[2], x[3]);
            reinterpret_cast<float4*>(d)[1] = make_float4(x[4], x[5], x[6], x[7]);
          } else {
            #pragma unroll
            for (int q = 0; q < 8; ++q)
              if (e0 + q < cols) d[q] = x[q];
          }
        }
      }
    }
    __syncthreads();
  }
}

struct Identity {
  __device__ __forceinline__ float operator()(int, int, float v) const { return v; }
};

// load_tile for an f32 or bf16 source (f32 values are rounded to bf16).
__device__ __forceinline__ void load_tile_any(const Tile& t, const void* __restrict__ src, long ld, int rows_valid,
                                              int cols_valid, bool src_bf16) {
  if (src_bf16) {
    load_tile(t, static_cast<const __nv_bfloat16*>(src), ld, rows_valid, cols_valid);
    return;
  }
  const float* s = static_cast<const float*>(src);
  const int chunks = t.cols / 8;
  const int total = t.rows * chunks;
  const bool vec_ok = ((reinterpret_cast<uintptr_t>(src) & 15) == 0) && ((ld & 3) == 0);
  // Four chunks per thread per pass: all loads are issued before any convert.
  constexpr int kBatch = 4;
  for (int it0 = threadIdx.x; it0 < total; it0 += kBatch * blockDim.x) {
    float f[kBatch][8];
#pragma unroll
    for (int q = 0; q < kBatch; ++q) {
      const int it = it0 + q * blockDim.x;
      const int r8 = it & 7;
      const int rest = it >> 3;
      const int j = rest % chunks;
      const int r = (rest / chunks) * 8 + r8;
      const int c0 = j * 8;
      if (it < total && r < rows_valid && vec_ok && c0 + 8 <= cols_valid) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(s + r * ld + c0));
        const float4 b = __ldg(reinterpret_cast<const float4*>(s + r * ld + c0 + 4));
        f[q][0] = a.x; f[q][1] = a.y; f[q][2] = a.z; f[q][3] = a.w;
        f[q][4] = b.x; f[q][5] = b.y; f[q][6] = b.z; f[q][7] = b.w;
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int c = c0 + e;
          f[q][e] = (it < total && r < rows_valid && c < cols_valid) ? __ldg(s + r * ld + c) : 0.f;
        }
      }
    }
#pragma unroll
    for (int q = 0; q < kBatch; ++q) {
      const int it = it0 + q * blockDim.x;
      if (it >= total) break;
      const int r8 = it & 7;
      const int rest = it >> 3;
      const int j = rest % chunks;
      const int r = (rest / chunks) * 8 + r8;
      tile_st16(t, r, j, pack8(f[q]));
    }
  }
}

// Copy a pre-arranged tile image (already in core-matrix order, `bytes` long,
// 16-byte aligned) from global memory, asynchronously like load_tile.
__device__ __forceinline__ void load_image(const Tile& t, const void* __restrict__ src, int bytes) {
  const uint8_t* s = static_cast<const uint8_t*>(src);
  for (int i = threadIdx.x; i < bytes / 16; i += blockDim.x) cp_async16(t.saddr + i * 16, s + i * 16);
}

__device__ __forceinline__ void zero_tile(const Tile& t) {
  for (int i = threadIdx.x; i < t.rows * t.cols / 8; i += blockDim.x)
    st_shared_v4(t.saddr + i * 16, make_uint4(0, 0, 0, 0));
}

// Block-wide sum; `scratch` holds >= 32 floats.
__device__ __forceinline__ float block_sum(float v, float* scratch) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) scratch[threadIdx.x >> 5] = v;
  __syncthreads();
  float s = 0.f;
  for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) s += scratch[w];
  __syncthreads();
  return s;
}

// Sum / max of a per-thread value over the kParts threads that own one row;
// `pair` holds kThreads floats of shared memory.
__device__ __forceinline__ float row_pair_sum(float v, float* pair) {
  __syncthreads();
  pair[threadIdx.x] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < kParts; ++j) s += pair[my_row() + kTile * j];
  __syncthreads();
  return s;
}
__device__ __forceinline__ float row_pair_max(float v, float* pair) {
  __syncthreads();
  pair[threadIdx.x] = v;
  __syncthreads();
  float s = -INFINITY;
#pragma unroll
  for (int j = 0; j < kParts; ++j) s = fmaxf(s, pair[my_row() + kTile * j]);
  __syncthreads();
  return s;
}

// ------------------------------------------------------------------ CTA context

// Barrier after the staging loads of a kernel's prologue: this thread's
// cp.async copies have landed, all threads' tiles are visible to every thread
// and to the tensor core, and TMEM allocation is ordered before later use.
__device__ __forceinline__ void tiles_ready() {
  cp_async_wait_all();
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
}

// Per-CTA MMA context: TMEM base, one completion barrier and its parity.
struct MmaCtx {
  uint64_t* bar;
  uint32_t tmem;
  uint32_t phase;
  bool ok;

  // Everybody: make staged operands visible, then thread 0 issues `issue()`,
  // commits, and all threads wait for completion.
  template <class F>
  __device__ __forceinline__ void run(F issue) {
    cp_async_wait_all();
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (threadIdx.x == 0 && ok) {
      issue();
      mma_commit(bar);
    }
    if (ok) ok = mbar_wait(bar, phase, kErrMmaTimeout);
    phase ^= 1u;
    tc_fence_after();
  }

  // As run(), but this thread's newest committed cp.async group may stay in
  // flight (it must not feed this MMA).
  template <class F>
  __device__ __forceinline__ void run_keep_newest(F issue) {
    cp_async_wait_group<1>();
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (threadIdx.x == 0 && ok) {
      issue();
      mma_commit(bar);
    }
    if (ok) ok = mbar_wait(bar, phase, kErrMmaTimeout);
    phase ^= 1u;
    tc_fence_after();
  }
};

}  // namespace ts
