// Forward of the multi-view chunked scan (reference scan_chunk.linattn_views,
// src/thetascan/_core/ops/scan_chunk.py:246-339), in three kernels:
//   1. scan_state_kernel   per tile: dS_r = k^T (u_r * v)          (tcgen05)
//   2. scan_prefix_kernel  per (b,h,r): exclusive scan of the tile states
//                           S_in(n) = e^{128 la} S_in(n-1) + dS(n-1)  (f32)
//   3. scan_out_kernel     per tile: score q.k^T once, then per retention
//                           out_r = (w_r o causal o score) v + (c_r q) S_in  (tcgen05)
// Tile kernels run kThreads = 512 threads: the kParts threads of token row r
// (r, r+128, ...) split its columns into 16-column chunks.  A stale slot
// (weights 1 - alpha^(t-j)) is carried with its auxiliary decayed slot (see
// scan.cuh).
#include "capi_internal.h"
#include "scan.cuh"

namespace ts {

// ------------------------------------------------------------------ 1. tile states

__global__ void __launch_bounds__(kThreads) scan_state_kernel(ScanParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint64_t bar;
  __shared__ uint32_t tmem_base;
  const int n = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int row = my_row(), part = my_part(), quad = my_quad();
  const int warp = threadIdx.x >> 5;
  const int t0 = n * kTile;
  const int rows = min(kTile, p.T - t0);

  const uint32_t base = smem_u32(smem);
  Tile tk{base, kTile, p.DkM};
  Tile tv{tk.saddr + kTile * p.DkM * 2, kTile, p.DvP};
  Tile tw{tv.saddr + kTile * p.DvP * 2, kTile, p.DvP};

  const int mblocks = p.DkM / kTile;
  const int cols_needed = mblocks * p.DvP;
  const uint32_t ncols = cols_needed <= 32 ? 32 : cols_needed <= 64 ? 64 : cols_needed <= 128 ? 128
                         : cols_needed <= 256 ? 256 : 512;

  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(&tmem_base, ncols);

  const __nv_bfloat16* kp = p.k + b * p.ks[0] + h * p.ks[1] + static_cast<long long>(t0) * p.ks[2];
  const __nv_bfloat16* vp = p.v + b * p.vs[0] + h * p.vs[1] + static_cast<long long>(t0) * p.vs[2];
  load_tile(tk, kp, p.ks[2], rows, p.Dk);
  load_payload(p, tv, vp, rows);

  tiles_ready();
  MmaCtx ctx{&bar, tmem_base, 0u, true};

  // One slot at a time through one TMEM region: the update, then its store
  // (accumulator row of block mb is feature mb*128 + row; states are stored
  // value-major, [DvP][DkM], so lanes of a warp write consecutive features).
  for (int r = 0; r < p.R; ++r) {
    const float la = head_la(p, r, h);
    // u_r(j): this tile's key weights in the leaving state.
    const float u = slot_key_weight(p, r, la, rows, row);
    for (int j = part; j < p.DvP / 8; j += kParts) {
      float f[8];
      unpack8(tile_ld16(tv, row, j), f);
#pragma unroll
      for (int e = 0; e < 8; ++e) f[e] *= u;
      tile_st16(tw, row, j, pack8(f));
    }
    ctx.run([&] {
      for (int mb = 0; mb < mblocks; ++mb) {
        const uint32_t d = ctx.tmem + static_cast<uint32_t>(mb * p.DvP);
        gemm_issue(d, mnmajor(tk, 0, mb * kTile), mnmajor(tw), p.DvP, kTile, false);
      }
    });
    float* dst_base = p.states + state_index(p, b, h, n, r) * p.DkM * p.DvP;
    for (int mb = 0; mb < mblocks; ++mb) {
      float* dst = dst_base + mb * kTile + row;
      for (int c = 16 * part; c < p.DvP; c += kChunkStep) {
        float v[16];
        tmem_ld16(tmem_addr(ctx.tmem, quad * 32, mb * p.DvP + c), v);
#pragma unroll
        for (int e = 0; e < 16; ++e) dst[static_cast<size_t>(c + e) * p.DkM] = v[e];
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem_base, ncols);
}

// ------------------------------------------------------------------ 2. prefix over tiles

// The lane of a stale slot X carries its auxiliary slot a too:
//   S_X(n+1) = S_X(n) + (1 - C_n) S_a(n) + dS_X(n),  S_a(n+1) = C_n S_a(n) + dS_a(n)
// from zero states (stale slots take no boundary states).
__device__ __forceinline__ void stale_prefix(const ScanParams& p, const PrefixLane& l) {
  const int a = p.partner[l.r];
  const float la = head_la(p, l.r, l.h);
  const float closing = __expf(la * static_cast<float>(kTile));
  const float closing_last = __expf(la * static_cast<float>(tile_len(p, p.NT - 1)));
  const float open = one_minus_exp(la * static_cast<float>(kTile));
  const float open_last = one_minus_exp(la * static_cast<float>(tile_len(p, p.NT - 1)));
  const bool in_image = l.f8 * 8 < p.DkP;
  const size_t img_off = static_cast<size_t>(l.f8) * p.DvP * 16 + static_cast<size_t>(l.c) * 16;
  const size_t elem = static_cast<size_t>(l.c) * p.DkM + l.f8 * 8;
  float X[8], A[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) X[e] = A[e] = 0.f;
  constexpr int kB = kPrefixBatch / 2;
  const int last_used = p.NT - 1;
  auto store8 = [&](int slot, int n, const float* S) {
    const size_t si = state_index(p, l.b, l.h, n, slot);
    float4* ptr = reinterpret_cast<float4*>(p.states + si * p.DkM * p.DvP + elem);
    ptr[0] = make_float4(S[0], S[1], S[2], S[3]);
    ptr[1] = make_float4(S[4], S[5], S[6], S[7]);
    if (in_image) {
      uint8_t* img = reinterpret_cast<uint8_t*>(p.images) + si * static_cast<size_t>(image_bytes(p)) + img_off;
      *reinterpret_cast<uint4*>(img) = pack8(S);
    }
  };
  for (int n0 = 0; n0 < p.NT; n0 += kB) {
    float4 ux[kB][2], ua[kB][2];
#pragma unroll
    for (int k = 0; k < kB; ++k) {
      const int n = n0 + k;
      ux[k][0] = ux[k][1] = ua[k][0] = ua[k][1] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (n < last_used) {
        const float4* px = reinterpret_cast<const float4*>(
            p.states + state_index(p, l.b, l.h, n, l.r) * p.DkM * p.DvP + elem);
        const float4* pa = reinterpret_cast<const float4*>(
            p.states + state_index(p, l.b, l.h, n, a) * p.DkM * p.DvP + elem);
        ux[k][0] = px[0];
        ux[k][1] = px[1];
        ua[k][0] = pa[0];
        ua[k][1] = pa[1];
      }
    }
#pragma unroll
    for (int k = 0; k < kB; ++k) {
      const int n = n0 + k;
      if (n >= p.NT) break;
      store8(l.r, n, X);
      store8(a, n, A);
      const float cl = n + 1 < p.NT ? closing : closing_last;
      const float op = n + 1 < p.NT ? open : open_last;
      const float vx[8] = {ux[k][0].x, ux[k][0].y, ux[k][0].z, ux[k][0].w,
                           ux[k][1].x, ux[k][1].y, ux[k][1].z, ux[k][1].w};
      const float va[8] = {ua[k][0].x, ua[k][0].y, ua[k][0].z, ua[k][0].w,
                           ua[k][1].x, ua[k][1].y, ua[k][1].z, ua[k][1].w};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        X[e] = X[e] + op * A[e] + vx[e];
        A[e] = A[e] * cl + va[e];
      }
    }
  }
}

__global__ void __launch_bounds__(256) scan_prefix_kernel(ScanParams p) {
  const PrefixLane l = prefix_lane(p);
  if (!l.active) return;
  if (p.kind[l.r] == kSlotAux) return;   // carried by its stale slot's lane
  if (p.kind[l.r] == kSlotStale) {
    stale_prefix(p, l);
    return;
  }
  const float la = head_la(p, l.r, l.h);
  const bool decayed = p.la[l.r] != nullptr;
  const float closing = decayed ? __expf(la * static_cast<float>(kTile)) : 1.f;
  const float closing_last = decayed ? __expf(la * static_cast<float>(tile_len(p, p.NT - 1))) : 1.f;
  const bool in_image = l.f8 * 8 < p.DkP;
  const size_t img_off = static_cast<size_t>(l.f8) * p.DvP * 16 + static_cast<size_t>(l.c) * 16;
  const size_t elem = static_cast<size_t>(l.c) * p.DkM + l.f8 * 8;
  // S_in(0): the initial state, or zero.
  float S[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const int f = l.f8 * 8 + e;
    S[e] = (p.init != nullptr && f < p.Dk && l.c < p.Dv) ? __ldg(p.init + boundary_index(p, l.b, l.h, l.r, f, l.c))
                                                       : 0.f;
  }
  // Loads of a batch of tiles are issued together (the in-place writes of a
  // batch touch only tiles whose values were already read), so the serial
  // chain pays one memory latency per batch rather than per tile.  The last
  // tile's state only matters for the final state (all_tiles).
  const int last_used = p.all_tiles ? p.NT : p.NT - 1;
  for (int n0 = 0; n0 < p.NT; n0 += kPrefixBatch) {
    float4 u[kPrefixBatch][2];
#pragma unroll
    for (int k = 0; k < kPrefixBatch; ++k) {
      const int n = n0 + k;
      u[k][0] = u[k][1] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (n < last_used) {
        const float4* ptr = reinterpret_cast<const float4*>(
            p.states + state_index(p, l.b, l.h, n, l.r) * p.DkM * p.DvP + elem);
        u[k][0] = ptr[0];
        u[k][1] = ptr[1];
      }
    }
#pragma unroll
    for (int k = 0; k < kPrefixBatch; ++k) {
      const int n = n0 + k;
      if (n >= p.NT) break;
      const size_t si = state_index(p, l.b, l.h, n, l.r);
      if (p.store) {
        float4* ptr = reinterpret_cast<float4*>(p.states + si * p.DkM * p.DvP + elem);
        ptr[0] = make_float4(S[0], S[1], S[2], S[3]);
        ptr[1] = make_float4(S[4], S[5], S[6], S[7]);
        if (in_image) {
          uint8_t* img = reinterpret_cast<uint8_t*>(p.images) + si * static_cast<size_t>(image_bytes(p)) + img_off;
          *reinterpret_cast<uint4*>(img) = pack8(S);
        }
      }
      const float cl = n + 1 < p.NT ? closing : closing_last;
      const float v[8] = {u[k][0].x, u[k][0].y, u[k][0].z, u[k][0].w, u[k][1].x, u[k][1].y, u[k][1].z, u[k][1].w};
#pragma unroll
      for (int e = 0; e < 8; ++e) S[e] = S[e] * cl + v[e];
    }
  }
  if (p.final_state != nullptr && l.c < p.Dv) {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int f = l.f8 * 8 + e;
      if (f < p.Dk) p.final_state[boundary_index(p, l.b, l.h, l.r, f, l.c)] = S[e];
    }
  }
}

// ------------------------------------------------------------------ 3. tile outputs

__global__ void __launch_bounds__(kThreads) scan_out_kernel(ScanParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint64_t bar;
  __shared__ uint32_t tmem_base;
  const int n = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int row = my_row(), part = my_part(), quad = my_quad();
  const int warp = threadIdx.x >> 5;
  const int t0 = n * kTile;
  const int rows = min(kTile, p.T - t0);

  const uint32_t base = smem_u32(smem);
  Tile tq{base, kTile, p.DkP};
  Tile tk{tq.saddr + kTile * p.DkP * 2, kTile, p.DkP};
  Tile tp{tk.saddr + kTile * p.DkP * 2, kTile, kTile};
  Tile tv{tp.saddr + kTile * kTile * 2, kTile, p.DvP};
  Tile ts{tv.saddr + kTile * p.DvP * 2, p.DvP, p.DkP};
  __shared__ float decay[4 * kTile];
  fill_decay(p, h, decay);

  // Fold mode (payloads up to a tile wide): q is loaded once and stays
  // unscaled.  A slot's read is P_r v + q S_r with carry 1 (plain sum, the
  // stale slot's own state) straight into its accumulator, and the decayed
  // cross term c_r(i) (q S_r) -- or the stale slot's (1 - c(i)) (q S_a) -- in
  // a second accumulator scaled per row on the way out.  Each slot is stored
  // right after its products (the P tile doubles as the store stage), and the
  // next slot's state image streams into the key tile's region, free after
  // the score, meanwhile.
  const bool fold = p.DvP <= kTile && kTile + 2 * p.DvP <= 512;
  const int cols_needed = fold ? kTile + 2 * p.DvP : kTile + p.RU * p.DvP;
  const uint32_t ncols = cols_needed <= 256 ? 256 : 512;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(&tmem_base, ncols);

  const __nv_bfloat16* qp = p.q + b * p.qs[0] + h * p.qs[1] + static_cast<long long>(t0) * p.qs[2];
  const __nv_bfloat16* kp = p.k + b * p.ks[0] + h * p.ks[1] + static_cast<long long>(t0) * p.ks[2];
  const __nv_bfloat16* vp = p.v + b * p.vs[0] + h * p.vs[1] + static_cast<long long>(t0) * p.vs[2];
  const bool cross_any = n > 0 || p.init != nullptr;
  auto image_at = [&](int slot) {
    return reinterpret_cast<const uint8_t*>(p.images) +
           state_index(p, b, h, n, slot) * static_cast<size_t>(image_bytes(p));
  };
  load_tile(tq, qp, p.qs[2], rows, p.Dk);
  load_tile(tk, kp, p.ks[2], rows, p.Dk);
  load_payload(p, tv, vp, rows);
  if (fold && cross_any) load_image(ts, image_at(0), image_bytes(p));

  tiles_ready();
  MmaCtx ctx{&bar, tmem_base, 0u, true};
  const uint32_t t_score = ctx.tmem;
  ctx.run([&] { gemm_issue(t_score, kmajor(tq), kmajor(tk), kTile, p.DkP, false); });

  if (fold) {
    const Tile img[2] = {ts, Tile{tk.saddr, p.DvP, p.DkP}};
    const uint32_t c_out = kTile, c_x = kTile + p.DvP;
    float* stage = reinterpret_cast<float*>(smem + (tp.saddr - base));
    const size_t row0 = ((static_cast<size_t>(b) * p.H + h) * p.T + t0) * p.Dv;
    for (int r = 0; r < p.RU; ++r) {
      const float la = head_la(p, r, h);
      const bool decayed = p.la[r] != nullptr;
      const bool stale = p.kind[r] == kSlotStale;
      // image r+1 into the buffer slot r-1 read (its products are done)
      if (cross_any && r + 1 < p.RU) load_image(img[(r + 1) & 1], image_at(r + 1), image_bytes(p));
      cp_async_commit();
      for (int c = 16 * part; c < kTile; c += kChunkStep) {
        float sc[16], f[16];
        tmem_ld16(tmem_addr(t_score, quad * 32, c), sc);
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const int j = c + e;
          f[e] = (j <= row) ? decay[r * kTile + row - j] * sc[e] : 0.f;
        }
        tile_st16(tp, row, c / 8, pack8(f));
        tile_st16(tp, row, c / 8 + 1, pack8(f + 8));
      }
      const Tile& im = img[r & 1];
      // the carry-1 state (plain sum, stale) accumulates into the read itself
      const bool direct = cross_any && (!decayed || stale);
      const bool scaled = cross_any && decayed && !stale;
      ctx.run_keep_newest([&] {
        gemm_issue(ctx.tmem + c_out, kmajor(tp), mnmajor(tv), p.DvP, kTile, false);
        if (direct) gemm_issue(ctx.tmem + c_out, kmajor(tq), kmajor(im), p.DvP, p.DkP, true);
        if (scaled) gemm_issue(ctx.tmem + c_x, kmajor(tq), kmajor(im), p.DvP, p.DkP, false);
      });
      bool second = scaled;
      if (cross_any && stale) {
        // + (1 - c(i)) q S_a: the auxiliary image into the buffer just read
        load_image(im, image_at(p.partner[r]), image_bytes(p));
        ctx.run([&] { gemm_issue(ctx.tmem + c_x, kmajor(tq), kmajor(im), p.DvP, p.DkP, false); });
        second = true;
      }
      const float x = la * static_cast<float>(row + 1);
      const float row_scale = stale ? one_minus_exp(x) : __expf(x);
      void* dst = p.out_bf16 ? static_cast<void*>(reinterpret_cast<__nv_bfloat16*>(p.out[r]) + row0)
                             : static_cast<void*>(reinterpret_cast<float*>(p.out[r]) + row0);
      store_rows(ctx.tmem, c_out, p.DvP, p.Dv, rows, dst, p.Dv, p.out_bf16 != 0, stage, Identity{}, nullptr,
                 second ? static_cast<int>(c_x) : -1, row_scale);
    }
    cp_async_wait_all();
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem_base, ncols);
    return;
  }

  for (int r = 0; r < p.RU; ++r) {
    const float la = head_la(p, r, h);
    const bool decayed = p.la[r] != nullptr;
    const bool stale = p.kind[r] == kSlotStale;
    // P_r row: w(row, j) * score(row, j) on the causal triangle.
    for (int c = 16 * part; c < kTile; c += kChunkStep) {
      float s[16];
      tmem_ld16(tmem_addr(t_score, quad * 32, c), s);
      float f[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const int j = c + e;
        f[e] = (j <= row) ? decay[r * kTile + row - j] * s[e] : 0.f;
      }
      tile_st16(tp, row, c / 8, pack8(f));
      tile_st16(tp, row, c / 8 + 1, pack8(f + 8));
    }
    const bool cross = n > 0 || p.init != nullptr;
    auto image_of = [&](int slot) {
      return reinterpret_cast<const uint8_t*>(p.images) +
             state_index(p, b, h, n, slot) * static_cast<size_t>(image_bytes(p));
    };
    if (cross) {
      load_image(ts, image_of(r), image_bytes(p));
      // carry c(i) = e^{la (i+1)}; a stale slot reads its own state with weight 1
      const float carry_la = la;
      load_scaled_rows(tq, qp, p.qs[2], rows, p.Dk, -1, [&](int t) {
        return decayed && !stale ? __expf(carry_la * static_cast<float>(t + 1)) : 1.f;
      });
    }
    const uint32_t t_out = ctx.tmem + static_cast<uint32_t>(kTile + r * p.DvP);
    ctx.run([&] {
      gemm_issue(t_out, kmajor(tp), mnmajor(tv), p.DvP, kTile, false);
      if (cross) gemm_issue(t_out, kmajor(tq), kmajor(ts), p.DvP, p.DkP, true);
    });
    if (cross && stale) {
      // + (1 - c(i)) q S_a: the auxiliary state, whose weights have not yet
      // reached the stale ones by the distance i + 1 into this tile
      load_image(ts, image_of(p.partner[r]), image_bytes(p));
      const float carry_la = la;
      load_scaled_rows(tq, qp, p.qs[2], rows, p.Dk, -1, [&](int t) {
        return one_minus_exp(carry_la * static_cast<float>(t + 1));
      });
      ctx.run([&] { gemm_issue(t_out, kmajor(tq), kmajor(ts), p.DvP, p.DkP, true); });
    }
  }

  // Coalesced stores through a stage on the (now idle) P tile.
  float* stage = reinterpret_cast<float*>(smem + (tp.saddr - base));
  for (int r = 0; r < p.RU; ++r) {
    const size_t row0 = ((static_cast<size_t>(b) * p.H + h) * p.T + t0) * p.Dv;
    void* dst = p.out_bf16 ? static_cast<void*>(reinterpret_cast<__nv_bfloat16*>(p.out[r]) + row0)
                           : static_cast<void*>(reinterpret_cast<float*>(p.out[r]) + row0);
    store_rows(ctx.tmem, kTile + r * p.DvP, p.DvP, p.Dv, rows, dst, p.Dv, p.out_bf16 != 0, stage, Identity{});
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem_base, ncols);
}

// ------------------------------------------------------------------ host launch

size_t scan_state_smem(const ScanParams& p) { return static_cast<size_t>(kTile) * (p.DkM + 2 * p.DvP) * 2; }
size_t scan_out_smem(const ScanParams& p) {
  return static_cast<size_t>(kTile) * (2 * p.DkP + kTile + p.DvP) * 2 + static_cast<size_t>(p.DvP) * p.DkP * 2;
}

int launch_scan_chain(const ScanParams& p, cudaStream_t s);

// The forward kernels; `tile_states` / `outputs` select the parts that run
// (the stages of a sequence shard run them separately).  The carried states
// come from the TMEM-resident chain (scan_chain.cu) where it applies -- it
// recomputes every tile's update from k and v, so a stage-2 call does not
// need stage 1's tile updates -- else from the per-tile updates and the
// tile prefix below.
int launch_scan_fwd(const ScanParams& p, cudaStream_t s, bool tile_states, bool outputs) {
  const size_t sm1 = scan_state_smem(p), sm3 = scan_out_smem(p);
  cudaFuncSetAttribute(scan_state_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(sm1));
  cudaFuncSetAttribute(scan_out_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(sm3));
  const int chained = launch_scan_chain(p, s);
  if (chained < 0) return -chained;
  if (chained == 0) {
    const int state_tiles = p.all_tiles ? p.NT : p.NT - 1;
    if (tile_states && state_tiles > 0) {
      scan_state_kernel<<<dim3(state_tiles, p.H, p.B), kThreads, sm1, s>>>(p);
      if (int e = check_launch("scan_state_kernel")) return e;
    }
    // One serial chain per state element: the forward chain streams one input
    // and two outputs per tile at about half of HBM bandwidth already (a
    // two-level version, measured, was slower for its second read of the tile
    // states); the backward's three inputs per tile take the two-level form.
    scan_prefix_kernel<<<prefix_grid(p.DkM, p.DvP, p.R, p.B * p.H), 256, 0, s>>>(p);
    if (int e = check_launch("scan_prefix_kernel")) return e;
  }
  if (!outputs) return 0;
  scan_out_kernel<<<dim3(p.NT, p.H, p.B), kThreads, sm3, s>>>(p);
  return check_launch("scan_out_kernel");
}

}  // namespace ts
