// Reverse tile chain of the scan backward: one CTA per (batch, head) walks
// the tiles from the last to the first with the gradient of every slot's
// carried state, G, resident in tensor memory (f32):
//   G(NT-1) = dfinal (or 0),   G(n-1) = C_n G(n) + dSloc(n),
//   dSloc(n) = sum_t c(i) q_t^T dout_t                    (tcgen05, into G)
// the reverse of the forward recursion S_in(n+1) = C_n S_in(n) + dS(n)
// (reference scan_chunk.py:170-212).  Per tile it writes the bf16 image of
// G(n) that the dq/dk and dv kernels read, and for a decayed slot it adds two
// terms of the log-retention gradient,
//   carry    <S_in(n), sum_t (i+1) c(i) q_t^T dout_t>     (a second product,
//            one 128-feature block at a time into a scratch TMEM block,
//            against the forward's f32 S_in(n))
//   closing  len_n C_n <G(n), S_in(n)>,
// while the key-weight term <G(n), B'(n)> is formed by the dv kernel from its
// per-row cross products (ScanGradParams.key_dla_in_dv).  It replaces the
// per-tile local-term kernel and the HBM reverse prefix (f32 dSloc written,
// re-read and rewritten per tile) where it applies: no stale slots, the whole
// backward in one call (stage 0), payloads of whole 64-column boxes plus up
// to two extra columns and at most 128 wide.
//
// Operands: q tiles by TMA (128-byte swizzle, this GPU's memory, no
// multicast) through a two-stage ring; every slot's raw dout rows by one
// untiled bulk copy per tile; the epilogue forms each slot's weighted row
// operand c(i) dout (rounded to bf16) and, for the carry term first, (i+1)
// times that rounded row, in the swizzled MN-major layout the tensor core
// reads, in the slot's operand buffer.  The slots are interleaved: slot r's
// dSloc product runs while the epilogue works on slot r + 1.
//
// Where the (batch, head) CTAs would leave SMs idle, the slots are split
// over several CTAs of the same (batch, head), as in the forward chain.
//
// Warp roles (288 threads): warp 0 lane 0 issues the copies and the MMAs;
// warps 1-8 (two per TMEM lane quadrant, each taking half of every row's
// chunks) form operands and read G.  Every
// wait is bounded; a wait that gives up records a device error, and the CTA
// drains its copies and MMAs in flight before freeing TMEM.
#include "capi_internal.h"
#include "scan.cuh"
#include "tma.cuh"

namespace ts {

namespace {

// warp 0: copies and MMAs; warps 1-8: the epilogue, two warps per TMEM lane
// quadrant, each taking half of every row's chunks
constexpr int kBwdEpiWarps = 8;
constexpr int kBwdChainThreads = 32 * (1 + kBwdEpiWarps);

struct BwdChainLayout {
  int qboxes, vboxes;
  uint32_t q_bytes;        // one q tile: DkM / 64 swizzled boxes (two, a ring)
  uint32_t op_bytes;       // one slot's row operand: swizzled boxes + 16-column unit tile
  uint32_t raw_bytes;      // one slot's raw dout rows (128 x Dv bf16, 16-byte multiple)
  uint32_t off_op, off_raw, total;
};

__host__ __device__ inline uint32_t align_up(uint32_t x, uint32_t a) { return (x + a - 1) / a * a; }

__host__ __device__ inline BwdChainLayout bwd_chain_layout(int DkM, int Dv, int v_unit, int R) {
  BwdChainLayout L;
  L.qboxes = DkM / 64;
  L.vboxes = (Dv - v_unit) / 64;
  L.q_bytes = L.qboxes * kSwBox;
  L.op_bytes = L.vboxes * kSwBox + (v_unit ? kTile * 16 * 2 : 0);
  L.raw_bytes = align_up(static_cast<uint32_t>(kTile * Dv * 2), 16);
  L.off_op = 2 * L.q_bytes;                // 1024-aligned
  L.off_raw = L.off_op + R * L.op_bytes;   // 1024-aligned (op_bytes is)
  L.total = L.off_raw + R * L.raw_bytes;
  return L;
}

__device__ __forceinline__ uint32_t bwd_chain_tmem_cols(int n) {
  return n <= 32 ? 32u : n <= 64 ? 64u : n <= 128 ? 128u : n <= 256 ? 256u : 512u;
}

struct BwdChainShared {
  // Each barrier runs at most one phase ahead of every thread that waits on
  // it, so parity waits are exact:
  uint64_t load_q[2];                 // q ring stage s holds its tile
  uint64_t load_raw;                  // the tile's raw dout rows of every slot landed
  uint64_t epi_x;                     // a carry operand is ready / the scratch block is free (128 arrivals)
  uint64_t mma_x;                     // a carry product is done
  uint64_t epi_g[TS_MAX_RETENTIONS];  // slot r's G pass is done and its dSloc operand ready
  uint64_t mma_g[TS_MAX_RETENTIONS];  // slot r's dSloc product is done
  uint32_t tmem;
  int abort;
};

// Row `row` of a weighted row operand: columns [0, dvv) from the raw dout
// row, each multiplied by `scale`, rounded to bf16 (and, with `times` != 1,
// multiplied by `times` and rounded again), into the swizzled boxes; the
// remaining v_unit columns into the unit tile.  Rows past the tile's end are
// zero.
// `half` selects the 16-byte chunks 4 half .. 4 half + 3 of every box (the
// unit tile belongs to half 0).
__device__ __forceinline__ void build_row_operand(uint32_t op, uint32_t raw_row, int dvv, int v_unit, int vboxes,
                                                  uint32_t unit_off, int row, bool valid, float scale,
                                                  float times, int half) {
  for (int i = 0; i < vboxes; ++i) {
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) {
      const int c8 = 4 * half + cc;
      float f[8];
      if (valid) {
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
          uint32_t w;
          asm volatile("ld.shared.b32 %0, [%1];" : "=r"(w) : "r"(raw_row + ((i * 64 + c8 * 8 + e) * 2)));
          const float2 x = unpack_bf16(w);
          float a = __bfloat162float(__float2bfloat16_rn(x.x * scale));
          float b2 = __bfloat162float(__float2bfloat16_rn(x.y * scale));
          f[e] = a * times;
          f[e + 1] = b2 * times;
        }
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = 0.f;
      }
      st_shared_v4(op + i * kSwBox + sw128_offset(row, c8), pack8(f));
    }
  }
  if (v_unit && half == 0) {
    float u[2] = {0.f, 0.f};
    if (valid) {
      uint32_t w;
      asm volatile("ld.shared.b32 %0, [%1];" : "=r"(w) : "r"(raw_row + dvv * 2));
      const float2 x = unpack_bf16(w);
      u[0] = __bfloat162float(__float2bfloat16_rn(x.x * scale)) * times;
      u[1] = v_unit >= 2 ? __bfloat162float(__float2bfloat16_rn(x.y * scale)) * times : 0.f;
    }
    // unit tile in core-matrix order (128 rows x 16 columns): row r's columns
    // 0-7 at r * 16, columns 8-15 at 2048 + r * 16
    st_shared_v4(op + unit_off + row * 16, make_uint4(pack_bf16(u[0], u[1]), 0u, 0u, 0u));
    st_shared_v4(op + unit_off + kTile * 16 + row * 16, make_uint4(0u, 0u, 0u, 0u));
  }
}

}  // namespace

__global__ void __launch_bounds__(kBwdChainThreads, 1)
    scan_bwd_chain_kernel(ScanParams p, ScanGradParams g, const __grid_constant__ CUtensorMap map_q) {
  constexpr int kMaxDvP = kTile;
  extern __shared__ uint8_t smem_raw[];
  __shared__ BwdChainShared sh;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.x / p.H, h = blockIdx.x % p.H;
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const int dvv = p.Dv - p.v_unit;
  // this CTA's slots: r0 .. r0 + nr - 1 (local index s = r - r0)
  const int grp = p.slot_group > 0 ? p.slot_group : p.R;
  const int r0 = blockIdx.y * grp, nr = min(grp, p.R - r0);
  const BwdChainLayout L = bwd_chain_layout(p.DkM, p.Dv, p.v_unit, grp);
  const int mblocks = p.DkM / kTile;
  const int region = mblocks * p.DvP;                  // TMEM columns of one slot's G
  const uint32_t t_x = static_cast<uint32_t>(grp * region);   // scratch block (one M block) after the G blocks
  const uint32_t ncols = bwd_chain_tmem_cols(grp * region + p.DvP);
  const int NT = p.NT;
  const int last_dla = g.dfinal != nullptr ? NT : NT - 1;   // tiles whose leaving state carries gradient
  auto local = [&](int n) { return n >= 1 || g.all_tiles; };
  auto want = [&](int r) { return p.la[r] != nullptr && g.dla[r] != nullptr; };

  if (threadIdx.x == 0) {
    mbar_init(&sh.load_q[0], 1);
    mbar_init(&sh.load_q[1], 1);
    mbar_init(&sh.load_raw, 1);
    mbar_init(&sh.epi_x, kBwdEpiWarps * 32);
    mbar_init(&sh.mma_x, 1);
    for (int r = 0; r < TS_MAX_RETENTIONS; ++r) {
      mbar_init(&sh.epi_g[r], kBwdEpiWarps * 32);
      mbar_init(&sh.mma_g[r], 1);
    }
    sh.abort = 0;
    fence_mbar_init();
    tma_prefetch_map(&map_q);
  }
  if (warp == 0) tmem_alloc(&sh.tmem, ncols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------------- copies + MMA
      // tiles are processed in the order k = 0 .. NT-1, tile n = NT-1-k
      auto issue_q = [&](int k) {
        const int n = NT - 1 - k;
        uint64_t* bar = &sh.load_q[k & 1];
        mbar_expect_tx(bar, L.q_bytes);
        for (int i = 0; i < L.qboxes; ++i)
          tma_load_4d(base + (k & 1) * L.q_bytes + i * kSwBox, &map_q, i * 64, n * kTile, h, b, bar);
      };
      auto issue_raw = [&](int k) {
        const int n = NT - 1 - k;
        const uint32_t bytes = static_cast<uint32_t>(tile_len(p, n) * p.Dv * 2);
        mbar_expect_tx(&sh.load_raw, bytes * nr);
        for (int s = 0; s < nr; ++s) {
          const __nv_bfloat16* src = g.dout[r0 + s] + ((static_cast<size_t>(b) * p.H + h) * p.T + n * kTile) * p.Dv;
          bulk_load(base + L.off_raw + s * L.raw_bytes, src, bytes, &sh.load_raw);
        }
      };
      const uint32_t id_v = idesc_bf16(kTile, 64 * L.vboxes, true, true);
      const uint32_t id_u = idesc_bf16(kTile, 16, true, true);
      // D (+)= q[:, block mb]^T . op: A = q^T (features x tokens), MN-major.
      auto product = [&](uint32_t qaddr, uint32_t d, int mb, uint32_t op, bool accumulate) {
#pragma unroll 1
        for (int ks = 0; ks < kTile / 16; ++ks) {
          const uint64_t ad = smem_desc_sw128(qaddr + 2 * mb * kSwBox + ks * 16 * kSwRow, kSwBox, kSwGroup);
          const uint64_t bd = smem_desc_sw128(op + ks * 16 * kSwRow, kSwBox, kSwGroup);
          const uint32_t acc = (accumulate || ks > 0) ? 1u : 0u;
          mma_bf16(d, ad, bd, id_v, acc);
          if (p.v_unit) {
            const uint64_t ud = smem_desc(op + L.vboxes * kSwBox + ks * 256, 128, kTile * 16);
            mma_bf16(d + 64 * L.vboxes, ad, ud, id_u, acc);
          }
        }
      };
      bool ok = true;
      int last_q[2] = {-1, -1}, raws = 0, nex = 0, nx = 0;
      int ng[TS_MAX_RETENTIONS] = {0, 0, 0, 0};
      issue_q(0);
      last_q[0] = 0;
      issue_raw(0);
      ++raws;
      if (NT > 1) {
        issue_q(1);
        last_q[1] = 1;
      }
      for (int k = 0; k < NT && ok; ++k) {
        const int n = NT - 1 - k;
        const uint32_t qaddr = base + (k & 1) * L.q_bytes;
        ok = mbar_wait(&sh.load_q[k & 1], (k >> 1) & 1, kErrCopyTimeout);   // the tile's q landed
        if (!ok) break;
        for (int s = 0; s < nr && ok; ++s) {
          const int r = r0 + s;
          const uint32_t op = base + L.off_op + s * L.op_bytes;
          if (want(r) && local(n)) {
            for (int mb = 0; mb < mblocks && ok; ++mb) {
              ok = mbar_wait(&sh.epi_x, nex & 1, kErrMmaTimeout);
              ++nex;
              if (!ok || *(volatile int*)&sh.abort) break;
              tc_fence_after();
              product(qaddr, tmem + t_x, mb, op, false);
              mma_commit(&sh.mma_x);
              ++nx;
            }
            if (!ok || *(volatile int*)&sh.abort) break;
          }
          ok = mbar_wait(&sh.epi_g[s], k & 1, kErrMmaTimeout);
          if (!ok || *(volatile int*)&sh.abort) break;
          tc_fence_after();
          if (local(n)) {
            for (int mb = 0; mb < mblocks; ++mb)
              product(qaddr, tmem + static_cast<uint32_t>(s * region + mb * p.DvP), mb, op, true);
            mma_commit(&sh.mma_g[s]);
            ++ng[s];
          }
          // every slot's raw rows are consumed once the last slot handed over
          if (s == nr - 1 && k + 1 < NT) {
            issue_raw(k + 1);
            ++raws;
          }
        }
        if (!ok || *(volatile int*)&sh.abort) break;
        if (k + 2 < NT) {
          // this q stage is free once the tile's last product has read it
          ok = mbar_wait(&sh.mma_g[nr - 1], (ng[nr - 1] - 1) & 1, kErrMmaTimeout);
          if (!ok) break;
          issue_q(k + 2);
          last_q[k & 1] = k + 2;
        }
      }
      if (!ok) *(volatile int*)&sh.abort = 1;
      // drain: every copy has landed and every product is done
      for (int st = 0; st < 2; ++st)
        if (last_q[st] >= 0) mbar_wait(&sh.load_q[st], (last_q[st] >> 1) & 1, kErrCopyTimeout);
      mbar_wait(&sh.load_raw, (raws - 1) & 1, kErrCopyTimeout);
      for (int s = 0; s < nr; ++s)
        if (ng[s] > 0) mbar_wait(&sh.mma_g[s], (ng[s] - 1) & 1, kErrMmaTimeout);
      if (nx > 0) mbar_wait(&sh.mma_x, (nx - 1) & 1, kErrMmaTimeout);
    }
  } else {
    // -------------------------------------------------------------------- epilogue
    const int quad = warp & 3;
    const int half = (warp - 1) >> 2;    // which of the two warps of this lane quadrant
    const int lrow = 32 * quad + lane;   // token row of the operands, feature row of a G block
    bool ok = true;
    int nx = 0;
    float acc[TS_MAX_RETENTIONS] = {0.f, 0.f, 0.f, 0.f};
    // G(NT-1): the gradient of the final state, or zero.
    for (int s = 0; s < nr; ++s)
      for (int mb = 0; mb < mblocks; ++mb) {
        const int r = r0 + s;
        const int f = mb * kTile + lrow;
        for (int c = 16 * half; c < p.DvP; c += 32) {
          float v[16];
#pragma unroll
          for (int e = 0; e < 16; ++e)
            v[e] = (g.dfinal != nullptr && f < p.Dk && c + e < p.Dv)
                       ? __ldg(g.dfinal + boundary_index(p, b, h, r, f, c + e)) : 0.f;
          tmem_st16(tmem_addr(tmem, 32 * quad, s * region + mb * p.DvP + c), v);
        }
      }
    for (int k = 0; k < NT && ok; ++k) {
      const int n = NT - 1 - k;
      const int len = tile_len(p, n);
      ok = mbar_wait(&sh.load_raw, k & 1, kErrCopyTimeout);
      if (!ok) break;
      for (int s = 0; s < nr && ok; ++s) {
        const int r = r0 + s;
        const bool decayed = p.la[r] != nullptr;
        const float la = head_la(p, r, h);
        const float c_row = decayed ? __expf(la * static_cast<float>(lrow + 1)) : 1.f;   // carry c(i), row i = lrow
        const uint32_t raw_row = base + L.off_raw + s * L.raw_bytes + lrow * p.Dv * 2;
        const uint32_t op = base + L.off_op + s * L.op_bytes;
        // G(n) of this slot is complete (and its operand buffer free) once the
        // previous tile's dSloc product of this slot is
        if (k > 0) ok = mbar_wait(&sh.mma_g[s], (k - 1) & 1, kErrMmaTimeout);
        if (!ok || *(volatile int*)&sh.abort) {
          ok = false;
          break;
        }
        tc_fence_after();
        const bool carry = want(r) && local(n);
        const bool closing_term = want(r) && n < last_dla;
        if (carry) {
          // (i+1) c(i) dout, from the bf16-rounded c(i) dout of dSloc's operand
          build_row_operand(op, raw_row, dvv, p.v_unit, L.vboxes, L.vboxes * kSwBox, lrow, lrow < len, c_row,
                            static_cast<float>(lrow + 1), half);
          fence_async_smem();
          tc_fence_before();
          mbar_arrive(&sh.epi_x);
        }
        // G(n): image out, log-retention terms, closing rescale; one
        // 128-feature block at a time (the carry product of a block in the
        // scratch block).
        const float closing = decayed ? __expf(la * static_cast<float>(len)) : 1.f;
        const float kc = static_cast<float>(len) * closing;
        const size_t si = state_index(p, b, h, n, r);
        const float* s_in = p.states + si * p.DkM * p.DvP;
        uint8_t* img = reinterpret_cast<uint8_t*>(g.gimages) + si * static_cast<size_t>(image_bytes(p));
        for (int mb = 0; mb < mblocks && ok; ++mb) {
          const int f = mb * kTile + lrow;
          const int f0 = f & ~7;
          // this warp's chunks of the row: kk = 2 i + par (every other chunk)
          const int par = (mb * (p.DvP / 16) + half) & 1;
          float sv[kMaxDvP / 2];
          if (carry || closing_term) {
            // every column of this warp's chunks in flight at once
#pragma unroll
            for (int i = 0; i < kMaxDvP / 32; ++i)
#pragma unroll
              for (int e = 0; e < 16; ++e) {
                const int c = 16 * (2 * i + par) + e;
                if (c < p.DvP) sv[16 * i + e] = s_in[static_cast<size_t>(c) * p.DkM + f];
              }
          }
          if (carry) {
            ok = mbar_wait(&sh.mma_x, nx & 1, kErrMmaTimeout);
            ++nx;
            if (!ok) break;
            tc_fence_after();
          }
          float part = 0.f;
#pragma unroll
          for (int i = 0; i < kMaxDvP / 32; ++i) {
            const int c = 16 * (2 * i + par);
            if (c >= p.DvP) break;
            const uint32_t ta = tmem_addr(tmem, 32 * quad, s * region + mb * p.DvP + c);
            float v[16];
            tmem_ld16(ta, v);
            if (carry) {
              float x[16];
              tmem_ld16(tmem_addr(tmem, 32 * quad, t_x + c), x);
#pragma unroll
              for (int e = 0; e < 16; ++e) part = fmaf(sv[16 * i + e], x[e], part);
            }
            if (closing_term) {
              float cg = 0.f;
#pragma unroll
              for (int e = 0; e < 16; ++e) cg = fmaf(sv[16 * i + e], v[e], cg);
              part = fmaf(kc, cg, part);
            }
            if (g.store) {
#pragma unroll
              for (int h8 = 0; h8 < 2; ++h8) {
                float x[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) x[e] = v[8 * h8 + e];
                transpose8(x);
                if (f0 < p.DkP)
                  *reinterpret_cast<uint4*>(img + static_cast<size_t>(f0 / 8) * p.DvP * 16 +
                                            static_cast<size_t>(c + 8 * h8 + (lane & 7)) * 16) = pack8(x);
              }
            }
            if (decayed && local(n)) {
#pragma unroll
              for (int e = 0; e < 16; ++e) v[e] *= closing;
              tmem_st16(ta, v);
            }
          }
          acc[r] += part;
          if (carry && mb + 1 < mblocks) {
            // the scratch block is free for the next block's carry product
            tc_fence_before();
            mbar_arrive(&sh.epi_x);
          }
        }
        if (!ok) break;
        // dSloc(n)'s row operand c(i) dout (the carry products are done)
        if (local(n))
          build_row_operand(op, raw_row, dvv, p.v_unit, L.vboxes, L.vboxes * kSwBox, lrow, lrow < len, c_row, 1.f,
                            half);
        fence_async_smem();
        tc_fence_before();
        mbar_arrive(&sh.epi_g[s]);
      }
    }
    if (!ok) *(volatile int*)&sh.abort = 1;
    // G(-1): the gradient of the initial state, after tile 0's dSloc products.
    if (ok && g.dinit != nullptr) {
      if (local(0))
        for (int s = 0; s < nr && ok; ++s) ok = mbar_wait(&sh.mma_g[s], (NT - 1) & 1, kErrMmaTimeout);
      tc_fence_after();
      if (ok) {
        for (int s = 0; s < nr; ++s)
          for (int mb = 0; mb < mblocks; ++mb) {
            const int r = r0 + s;
            const int f = mb * kTile + lrow;
            for (int c = 16 * half; c < p.DvP; c += 32) {
              float v[16];
              tmem_ld16(tmem_addr(tmem, 32 * quad, s * region + mb * p.DvP + c), v);
              if (f < p.Dk) {
#pragma unroll
                for (int e = 0; e < 16; ++e)
                  if (c + e < p.Dv) g.dinit[boundary_index(p, b, h, r, f, c + e)] = v[e];
              }
            }
          }
      }
    }
    for (int r = r0; r < r0 + nr; ++r) {
      if (!want(r)) continue;
      float v = acc[r];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0 && ok) atomicAdd(g.dla[r] + h, v);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, ncols);
}

// ------------------------------------------------------------------ host launch

size_t scan_bwd_chain_smem(const ScanParams& p) {
  const int grp = p.slot_group > 0 ? p.slot_group : p.R;
  return static_cast<size_t>(bwd_chain_layout(p.DkM, p.Dv, p.v_unit, grp).total) + 1024;
}

int chain_slot_group(const ScanParams& p);   // scan_chain.cu

// Runs the reverse chain where it applies; returns 1 if it ran, 0 if the
// caller should run the per-tile kernels and the HBM reverse prefix, or a
// negative TS_ERR_* code.
int launch_scan_bwd_chain(const ScanParams& pin, const ScanGradParams& g, cudaStream_t s) {
  ScanParams p = pin;
  const int dvv = p.Dv - p.v_unit;
  if (p.any_stale || p.R != p.RU || g.zero_start_final || !g.store) return 0;
  if (dvv % 64 != 0 || p.DvP != dvv + (p.v_unit ? 16 : 0) || p.DvP > kTile || p.Dv % 2 != 0) return 0;
  p.slot_group = chain_slot_group(p);
  if (p.slot_group * (p.DkM / kTile) * p.DvP + p.DvP > 512) return 0;
  // raw dout rows by untiled bulk copies: 16-byte aligned starts and lengths
  const long long len_last = p.T - static_cast<long long>(p.NT - 1) * kTile;
  if ((static_cast<long long>(p.T) * p.Dv * 2) % 16 != 0 || (len_last * p.Dv * 2) % 16 != 0) return 0;
  for (int r = 0; r < p.RU; ++r)
    if (reinterpret_cast<uintptr_t>(g.dout[r]) % 16 != 0) return 0;
  const size_t smem = scan_bwd_chain_smem(p);
  if (smem > 232448) return 0;
  CUtensorMap mq;
  const uint64_t dims[4] = {static_cast<uint64_t>(p.Dk), static_cast<uint64_t>(p.T), static_cast<uint64_t>(p.H),
                            static_cast<uint64_t>(p.B)};
  const int64_t strides[3] = {p.qs[2], p.qs[1], p.qs[0]};
  const uint32_t box[4] = {64u, static_cast<uint32_t>(kTile), 1u, 1u};
  if (!make_tmap_bf16_sw128(&mq, p.q, 4, dims, strides, box)) return 0;
  cudaFuncSetAttribute(scan_bwd_chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  scan_bwd_chain_kernel<<<dim3(p.B * p.H, ceil_div(p.R, p.slot_group)), kBwdChainThreads, smem, s>>>(p, g, mq);
  if (int e = check_launch("scan_bwd_chain_kernel")) return -e;
  return 1;
}

}  // namespace ts
