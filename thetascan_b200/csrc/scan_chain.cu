// Forward tile states of the multi-view scan as one sequential chain per
// (batch, head): the f32 state of every retention slot stays in tensor memory
// from the first tile to the last, so no per-tile update or carried state
// makes a round trip through HBM.  Per tile n and slot r, with
// C_n = e^{la_r len_n}:
//   S_in(n)  -> bf16 image and (decayed slots) f32 copy for the reads and the
//               backward, written straight from registers;
//   S <- C_n S_in(n)                                      (TMEM, in place)
//   S += k_n^T (u_r o [v_n | 1])                          (tcgen05, into S)
// which is the exclusive tile prefix of the reference chunk backend
// (src/thetascan/_core/ops/scan_chunk.py:170-212: per-tile update with the
// key weights of the leaving state, carried by the tile's closing factor),
// with 128-token tiles.  It replaces scan_state_kernel + scan_prefix_kernel
// (per-tile updates written to HBM, then an HBM-to-HBM prefix) wherever it
// applies: slots without a stale view, payload widths of whole 64-column
// boxes plus up to two unit columns, and states that fit the 512 TMEM columns.
//
// The slots are interleaved: slot r's update product of tile n runs while the
// epilogue writes out slot r + 1, and the key and payload tiles run through a
// two-stage load ring, so loads, products and the write-out overlap.  Where
// the (batch, head) CTAs would leave SMs idle, the slots are split over
// several CTAs of the same (batch, head) (chain_slot_group).  Warp
// roles (288 threads):
//   warp 0, lane 0  TMA loads (128-byte-swizzled boxes, tensor maps of this
//                   GPU's own memory, no multicast) and the tcgen05 MMA issue;
//   warps 1-8       epilogue, two warps per TMEM lane quadrant (warp w reads
//                   lanes 32 (w % 4) ..), splitting each row's chunks: each
//                   slot's weighted payload tile, the state write-out and the
//                   closing rescale.
// Every wait is bounded; a wait that gives up records a device error and the
// CTA drains its own copies and MMAs in flight before it frees TMEM and exits.
#include "capi_internal.h"
#include "scan.cuh"
#include "tma.cuh"

namespace ts {

namespace {

// warp 0: loads and MMAs; warps 1-8: the epilogue, two warps per TMEM lane
// quadrant, each taking every other 16-column chunk of a row
constexpr int kChainEpiWarps = 8;
constexpr int kChainThreads = 32 * (1 + kChainEpiWarps);

struct ChainLayout {
  int kboxes, vboxes;       // 64-column boxes of a key tile (DkM / 64) and a payload tile
  uint32_t k_bytes, v_bytes;
  uint32_t stage_bytes;     // one stage of the load ring: key tile, then payload tile
  uint32_t wv_bytes;        // one slot's weighted payload: swizzled boxes, then its unit tile
  uint32_t off_wv, total;   // byte offsets from the 1024-aligned base
};

__host__ __device__ inline ChainLayout chain_layout(int DkM, int dv_boxes, int v_unit, int R) {
  ChainLayout L;
  L.kboxes = DkM / 64;
  L.vboxes = dv_boxes;
  L.k_bytes = L.kboxes * kSwBox;
  L.v_bytes = L.vboxes * kSwBox;
  L.stage_bytes = L.k_bytes + L.v_bytes;
  L.wv_bytes = L.v_bytes + (v_unit ? kTile * 16 * 2 : 0);
  L.off_wv = 2 * L.stage_bytes;
  L.total = L.off_wv + R * L.wv_bytes;
  return L;
}

__device__ __forceinline__ uint32_t chain_tmem_cols(int n) {
  return n <= 32 ? 32u : n <= 64 ? 64u : n <= 128 ? 128u : n <= 256 ? 256u : 512u;
}

struct ChainShared {
  // Each barrier runs at most one phase ahead of every thread that waits on it.
  uint64_t full[2];                 // stage s holds its tile's key and payload rows
  uint64_t epi[TS_MAX_RETENTIONS];  // slot r of the tile is written out and its payload built (128 arrivals)
  uint64_t mma[TS_MAX_RETENTIONS];  // slot r's update product of the tile is complete
  uint32_t tmem;
  int abort;
};

}  // namespace

__global__ void __launch_bounds__(kChainThreads, 1)
    scan_chain_kernel(ScanParams p, const __grid_constant__ CUtensorMap map_k,
                      const __grid_constant__ CUtensorMap map_v) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ ChainShared sh;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.x / p.H, h = blockIdx.x % p.H;
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  // this CTA's slots: r0 .. r0 + nr - 1 (local index s = r - r0)
  const int grp = p.slot_group > 0 ? p.slot_group : p.R;
  const int r0 = blockIdx.y * grp, nr = min(grp, p.R - r0);
  const ChainLayout L = chain_layout(p.DkM, (p.Dv - p.v_unit) / 64, p.v_unit, grp);
  const int mblocks = p.DkM / kTile;
  const int region = mblocks * p.DvP;          // TMEM columns of one slot's state
  const uint32_t ncols = chain_tmem_cols(grp * region);
  const int NT = p.NT;

  if (threadIdx.x == 0) {
    mbar_init(&sh.full[0], 1);
    mbar_init(&sh.full[1], 1);
    for (int r = 0; r < TS_MAX_RETENTIONS; ++r) {
      mbar_init(&sh.epi[r], kChainEpiWarps * 32);
      mbar_init(&sh.mma[r], 1);
    }
    sh.abort = 0;
    fence_mbar_init();
    tma_prefetch_map(&map_k);
    tma_prefetch_map(&map_v);
  }
  if (warp == 0) tmem_alloc(&sh.tmem, ncols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------------- loads + MMA
      auto issue_load = [&](int n) {
        uint64_t* bar = &sh.full[n & 1];
        const uint32_t dst = base + (n & 1) * L.stage_bytes;
        mbar_expect_tx(bar, L.stage_bytes);
        for (int i = 0; i < L.kboxes; ++i) tma_load_4d(dst + i * kSwBox, &map_k, i * 64, n * kTile, h, b, bar);
        for (int i = 0; i < L.vboxes; ++i)
          tma_load_4d(dst + L.k_bytes + i * kSwBox, &map_v, i * 64, n * kTile, h, b, bar);
      };
      int last_load[2] = {-1, -1};
      int commits = 0;
      bool ok = true;
      for (int n = 0; n < 2 && n < NT; ++n) {
        issue_load(n);
        last_load[n] = n;
      }
      const uint32_t id_v = idesc_bf16(kTile, 64 * L.vboxes, true, true);
      const uint32_t id_u = idesc_bf16(kTile, 16, true, true);
      for (int n = 0; n < NT && ok; ++n) {
        const uint32_t kaddr = base + (n & 1) * L.stage_bytes;
        for (int s = 0; s < nr && ok; ++s) {
          ok = mbar_wait(&sh.epi[s], n & 1, kErrMmaTimeout);
          if (!ok || *(volatile int*)&sh.abort) break;
          tc_fence_after();
          const uint32_t wv = base + L.off_wv + s * L.wv_bytes;
          for (int mb = 0; mb < mblocks; ++mb) {
            const uint32_t d = tmem + static_cast<uint32_t>(s * region + mb * p.DvP);
#pragma unroll 1
            for (int ks = 0; ks < kTile / 16; ++ks) {
              // A = k^T (features x tokens): MN-major, 64-feature boxes LBO apart
              const uint64_t ad = smem_desc_sw128(kaddr + 2 * mb * kSwBox + ks * 16 * kSwRow, kSwBox, kSwGroup);
              const uint64_t bd = smem_desc_sw128(wv + ks * 16 * kSwRow, kSwBox, kSwGroup);
              mma_bf16(d, ad, bd, id_v, 1u);
              if (p.v_unit) {
                const uint64_t ud = smem_desc(wv + L.v_bytes + ks * 256, 128, kTile * 16);
                mma_bf16(d + 64 * L.vboxes, ad, ud, id_u, 1u);
              }
            }
          }
          mma_commit(&sh.mma[s]);
          ++commits;
        }
        if (!ok || *(volatile int*)&sh.abort) break;
        if (n + 2 < NT) {
          // stage n & 1 is free once the tile's last product has read the key
          // tile (commits complete in issue order; the epilogue consumed the
          // payload tile before it handed over)
          ok = mbar_wait(&sh.mma[nr - 1], n & 1, kErrMmaTimeout);
          if (!ok) break;
          issue_load(n + 2);
          last_load[n & 1] = n + 2;
        }
      }
      if (!ok) *(volatile int*)&sh.abort = 1;
      // Drain: every issued load has landed and every product is done before
      // the CTA frees its tensor memory and exits.
      for (int st = 0; st < 2; ++st)
        if (last_load[st] >= 0) mbar_wait(&sh.full[st], (last_load[st] >> 1) & 1, kErrCopyTimeout);
      if (commits > 0) {
        const int tiles_done = (commits + nr - 1) / nr;   // the last tile reached, partly or fully
        const int last_r = (commits - 1) % nr;
        mbar_wait(&sh.mma[last_r], (tiles_done - 1) & 1, kErrMmaTimeout);
      }
    }
  } else {
    // -------------------------------------------------------------------- epilogue
    const int quad = warp & 3;
    const int half = (warp - 1) >> 2;    // which of the two warps of this lane quadrant
    const int lrow = 32 * quad + lane;   // TMEM lane = token row of the payload tile = feature row of a state block
    const int nchunk = p.DvP / 16;       // 16-column chunks of a state block row
    bool ok = true;
    // S_in(0): the initial state, or zero.
    for (int s = 0; s < nr; ++s)
      for (int mb = 0; mb < mblocks; ++mb) {
        const int r = r0 + s;
        const int f = mb * kTile + lrow;
        for (int c = 16 * half; c < p.DvP; c += 32) {
          float v[16];
#pragma unroll
          for (int e = 0; e < 16; ++e)
            v[e] = (p.init != nullptr && f < p.Dk && c + e < p.Dv)
                       ? __ldg(p.init + boundary_index(p, b, h, r, f, c + e)) : 0.f;
          tmem_st16(tmem_addr(tmem, 32 * quad, s * region + mb * p.DvP + c), v);
        }
      }
    for (int n = 0; n < NT && ok; ++n) {
      const int len = tile_len(p, n);
      ok = mbar_wait(&sh.full[n & 1], (n >> 1) & 1, kErrCopyTimeout);
      if (!ok) break;
      const uint32_t vrow = base + (n & 1) * L.stage_bytes + L.k_bytes + lrow * kSwRow;
      for (int s = 0; s < nr && ok; ++s) {
        const int r = r0 + s;
        const bool decayed = p.la[r] != nullptr;
        const float la = head_la(p, r, h);
        // S_in(n) of this slot is complete (and its payload buffer free) once
        // the previous tile's product of this slot is
        if (n > 0) ok = mbar_wait(&sh.mma[s], (n - 1) & 1, kErrMmaTimeout);
        if (!ok || *(volatile int*)&sh.abort) {
          ok = false;
          break;
        }
        tc_fence_after();
        // Weighted payload u(j) [v_j | 1] (row j = lrow).  A swizzled row is
        // one 128-byte line whatever its chunk order, so the row scaling
        // ignores the swizzle; each lane walks its row's chunks from its own
        // starting chunk (row % 8), so the 8 lanes of a shared-memory phase
        // touch 8 different bank groups.
        const float u = slot_key_weight(p, r, la, len, lrow);
        const uint32_t wv = base + L.off_wv + s * L.wv_bytes;
        for (int i = 0; i < L.vboxes; ++i) {
          // this warp's four 16-byte chunks of the row (half 0: 0-3, half 1: 4-7)
          uint4 raw[4];
#pragma unroll
          for (int c = 0; c < 4; ++c) raw[c] = ld_shared_v4(vrow + i * kSwBox + (((4 * half + c) ^ (lrow & 7)) * 16));
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            float f8[8];
            unpack8(raw[c], f8);
#pragma unroll
            for (int e = 0; e < 8; ++e) f8[e] *= u;
            st_shared_v4(wv + i * kSwBox + lrow * kSwRow + (((4 * half + c) ^ (lrow & 7)) * 16), pack8(f8));
          }
        }
        if (p.v_unit && half == 0) {
          // unit tile (core-matrix order, 128 rows x 16 columns): columns 0
          // (and 1) are u(j), the rest zero
          const float w1 = p.v_unit >= 2 ? u : 0.f;
          st_shared_v4(wv + L.v_bytes + lrow * 16, make_uint4(pack_bf16(u, w1), 0u, 0u, 0u));
          st_shared_v4(wv + L.v_bytes + kTile * 16 + lrow * 16, make_uint4(0u, 0u, 0u, 0u));
        }
        fence_async_smem();
        // S_in(n) out (the image for the reads, an f32 copy of a decayed slot
        // for the backward), then the closing rescale in place.
        const float closing = decayed ? __expf(la * static_cast<float>(len)) : 1.f;
        const size_t si = state_index(p, b, h, n, r);
        float* st = p.states + si * p.DkM * p.DvP;
        uint8_t* img = reinterpret_cast<uint8_t*>(p.images) + si * static_cast<size_t>(image_bytes(p));
        for (int mb = 0; mb < mblocks; ++mb) {
          const int f = mb * kTile + lrow;
          const int f0 = f & ~7;
          for (int j = (mb * nchunk + half) & 1; j < nchunk; j += 2) {
            const int c = 16 * j;
            const uint32_t ta = tmem_addr(tmem, 32 * quad, s * region + mb * p.DvP + c);
            float v[16];
            tmem_ld16(ta, v);
            if (p.store) {
              if (decayed) {
#pragma unroll
                for (int e = 0; e < 16; ++e) st[static_cast<size_t>(c + e) * p.DkM + f] = v[e];
              }
#pragma unroll
              for (int h8 = 0; h8 < 2; ++h8) {
                float x[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) x[e] = v[8 * h8 + e];
                transpose8(x);   // lane l of the 8-group: column c + 8 h8 + l of features f0 .. f0 + 7
                if (f0 < p.DkP)
                  *reinterpret_cast<uint4*>(img + static_cast<size_t>(f0 / 8) * p.DvP * 16 +
                                            static_cast<size_t>(c + 8 * h8 + (lane & 7)) * 16) = pack8(x);
              }
            }
            if (decayed) {
#pragma unroll
              for (int e = 0; e < 16; ++e) v[e] *= closing;
              tmem_st16(ta, v);
            }
          }
        }
        tc_fence_before();
        mbar_arrive(&sh.epi[s]);
      }
    }
    if (!ok) *(volatile int*)&sh.abort = 1;
    // The final state, after the last tile's updates.
    if (ok && p.final_state != nullptr) {
      for (int s = 0; s < nr && ok; ++s) ok = mbar_wait(&sh.mma[s], (NT - 1) & 1, kErrMmaTimeout);
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
                  if (c + e < p.Dv) p.final_state[boundary_index(p, b, h, r, f, c + e)] = v[e];
              }
            }
          }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, ncols);
}

// ------------------------------------------------------------------ host launch

size_t scan_chain_smem(const ScanParams& p) {
  const ChainLayout L = chain_layout(p.DkM, (p.Dv - p.v_unit) / 64, p.v_unit, p.slot_group > 0 ? p.slot_group : p.R);
  return static_cast<size_t>(L.total) + 1024;
}

// Slots per chain CTA.  The chains are sequential over tiles, so a CTA's time
// is its slots' per-tile work: where the (batch, head) CTAs leave SMs idle,
// the slots are split into groups, one CTA each, as long as the whole grid
// still runs in one wave.
int chain_slot_group(const ScanParams& p) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int units = max(1, p.B * p.H);
  const int groups = max(1, min(p.R, sms / units));
  return ceil_div(p.R, groups);
}

// The chain runs where it applies (see the file comment) and the tensor maps
// of k and v can be expressed; returns 1 if it ran, 0 if the caller should
// run the tile-parallel kernels, or a TS_ERR_* code.
int launch_scan_chain(const ScanParams& pin, cudaStream_t s) {
  ScanParams p = pin;
  const int dvv = p.Dv - p.v_unit;
  if (p.any_stale || dvv % 64 != 0 || p.DvP != dvv + (p.v_unit ? 16 : 0)) return 0;
  p.slot_group = chain_slot_group(p);
  if (p.slot_group * (p.DkM / kTile) * p.DvP > 512) return 0;
  const size_t smem = scan_chain_smem(p);
  if (smem > 232448) return 0;
  CUtensorMap mk, mv;
  const uint64_t dims_k[4] = {static_cast<uint64_t>(p.Dk), static_cast<uint64_t>(p.T), static_cast<uint64_t>(p.H),
                              static_cast<uint64_t>(p.B)};
  const int64_t strides_k[3] = {p.ks[2], p.ks[1], p.ks[0]};
  const uint64_t dims_v[4] = {static_cast<uint64_t>(dvv), static_cast<uint64_t>(p.T), static_cast<uint64_t>(p.H),
                              static_cast<uint64_t>(p.B)};
  const int64_t strides_v[3] = {p.vs[2], p.vs[1], p.vs[0]};
  const uint32_t box[4] = {64u, static_cast<uint32_t>(kTile), 1u, 1u};
  if (!make_tmap_bf16_sw128(&mk, p.k, 4, dims_k, strides_k, box)) return 0;
  if (!make_tmap_bf16_sw128(&mv, p.v, 4, dims_v, strides_v, box)) return 0;
  cudaFuncSetAttribute(scan_chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  scan_chain_kernel<<<dim3(p.B * p.H, ceil_div(p.R, p.slot_group)), kChainThreads, smem, s>>>(p, mk, mv);
  if (int e = check_launch("scan_chain_kernel")) return -e;
  return 1;
}

}  // namespace ts
