// Shared definitions of the multi-view chunked scan kernels.
//
// Sequence tiles are 128 tokens.  For retention r with static per-head
// log-retention la (la = 0 for the plain sum) and local position i in a tile:
//   intra weight  w(i, j) = exp(la * (i - j))      (j <= i)
//   carry         c(i)    = exp(la * (i + 1))      (weight of the entering state)
//   key weight    u(j)    = exp(la * (127 - j))    (weight in the leaving state)
//   closing       exp(128 * la)                    (state decay across a tile)
// which is the tile algebra of the reference chunk backend
// (src/thetascan/_core/ops/scan_chunk.py:102-119, 170-212, 322-336) with a
// 128-token tile; every exponent is <= 0, so no reciprocal decay is formed.
//
// A stale slot reads with weights 1 - alpha^(t-j), the reference's stale view
// S_sum - S_fast (src/thetascan/_core/ops/interface.py:251-279), formed
// directly rather than as a difference of two reads (which would cancel for
// recent tokens, whose stale weight is near zero).  Its state S_X carries
// those weights; an auxiliary decayed slot a (same la, no output) carries
// S_a = the alpha-weighted state, and with C = e^{la len}:
//   intra weight  1 - e^{la (i - j)}
//   read          q S_X + (1 - c(i)) q S_a
//   key weight    1 - e^{la (len - 1 - j)}
//   recursion     S_X(n+1) = S_X(n) + (1 - C) S_a(n) + dS_X(n)
// so every weight is a nonnegative f32 number formed without cancellation.
#pragma once

#include "../../include/thetascan_b200.h"
#include "common.cuh"

namespace ts {

constexpr int kMaxSlots = 2 * TS_MAX_RETENTIONS;  // caller slots plus the auxiliary slots of stale ones
enum SlotKind : int { kSlotDecay = 0, kSlotStale = 1, kSlotAux = 2 };

struct ScanParams {
  int B, H, T;
  int Dk, Dv;     // logical widths (Dv includes the unit column)
  int DkP;        // Dk rounded up to 16 (MMA K of the score / read)
  int DkM;        // Dk rounded up to 128 (MMA M of the state update)
  int DvP;        // Dv rounded up to 16
  int NT, R;      // R: all slots; slots 0..RU-1 are the caller's, RU..R-1 auxiliary
  int RU;
  // chain kernels: slots per CTA (blockIdx.y selects the group of slots
  // [y * slot_group, ...)); 0 = all slots in one CTA
  int slot_group;
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  long long qs[3], ks[3], vs[3];
  int v_unit;                // the last v_unit (0..2) payload columns are the constant 1
  const float* la[kMaxSlots];   // nullptr = plain sum
  int kind[kMaxSlots];          // SlotKind
  int partner[kMaxSlots];       // stale slot <-> its auxiliary slot, else -1
  void* out[kMaxSlots];         // caller slots only
  int out_bf16;
  float* states;             // [B,H,NT,R,DkM,DvP] f32: dS, then S_in in place
  __nv_bfloat16* images;     // [B,H,NT,R] images of S_in (DvP rows x DkP cols)
  int any_stale;
  // Two-level reverse tile prefix of the backward (long sequences): NS
  // segments of kSegTiles tiles (NS = 0: one serial chain per state element).
  int NS;
  // sequence-shard boundary states, f32 [B,H,R,Dk,Dv] (payload column fastest)
  const float* init;         // state entering token 0, or null (zero)
  float* final_state;        // state after the last token (written), or null
  int all_tiles;             // tile states of every tile, the last one towards the final state
  int store;                 // the prefix writes S_in and images (0: final state only)
};

struct ScanGradParams {
  const __nv_bfloat16* dout[kMaxSlots];   // caller slots only
  void* dq;
  void* dk;
  void* dv;
  long long dvs[3];          // element strides of a [B,H,T,Dv - v_unit] view when dv_strided
  int dv_strided;
  int grad_bf16;
  float* dla[kMaxSlots];     // an auxiliary slot shares its stale slot's
  float* gstates;            // [B,H,NT,R,DkM,DvP] f32: local dS of every tile
  __nv_bfloat16* pstates;    // [B,H,NT,R,DkM,DvP] bf16: key-weight derivative of each tile's state
                             // (only ever dotted into the log-retention gradient)
  __nv_bfloat16* gimages;    // [B,H,NT,R] images of G (DvP rows x DkP cols)
  const float* dfinal;       // gradient of the final state (G of the last tile), or null
  float* dinit;              // gradient of the initial state (written), or null
  int all_tiles;             // local terms of every tile (the last one feeds the final state)
  int store;                 // the reverse prefix writes G, images and its log-retention terms
  int zero_start_final;      // dfinal is the gradient of the final state from a zero start
  float* gsegs;              // [B,H,R,NS,DkM,DvP] f32: segment totals of the reverse prefix (NS > 0)
  // The reverse chain (scan_bwd_chain.cu) ran: the dv kernel adds the
  // key-weight term of the log-retention gradient, <G_n, B'(n)>, from its
  // per-row cross products.
  int key_dla_in_dv;
};

__device__ __forceinline__ float head_la(const ScanParams& p, int r, int h) {
  return p.la[r] ? __ldg(p.la[r] + h) : 0.f;
}

__device__ __forceinline__ size_t state_index(const ScanParams& p, int b, int h, int n, int r) {
  return ((static_cast<size_t>(b) * p.H + h) * p.NT + n) * p.R + r;
}

__device__ __forceinline__ int image_bytes(const ScanParams& p) { return p.DvP * p.DkP * 2; }

// Tokens in tile n (the last tile may be ragged).
__device__ __forceinline__ int tile_len(const ScanParams& p, int n) { return min(kTile, p.T - n * kTile); }

// Weight of row j of a tile of `len` tokens in the state that leaves it,
// e^{la (len - 1 - j)} (1 for the plain sum), and 0 past the tile's end.
__device__ __forceinline__ float key_weight(float la, bool decayed, int len, int j) {
  if (j >= len) return 0.f;
  return decayed ? __expf(la * static_cast<float>(len - 1 - j)) : 1.f;
}

// 1 - e^{x} for x <= 0 without cancellation.
__device__ __forceinline__ float one_minus_exp(float x) { return -expm1f(x); }

// Key weight of slot r: the stale slot's is 1 - e^{la (len - 1 - j)}.
__device__ __forceinline__ float slot_key_weight(const ScanParams& p, int r, float la, int len, int j) {
  if (p.kind[r] == kSlotStale) return j < len ? one_minus_exp(la * static_cast<float>(len - 1 - j)) : 0.f;
  return key_weight(la, p.la[r] != nullptr, len, j);
}

// d/d la of slot r's key weight of row j.
__device__ __forceinline__ float slot_key_weight_dla(const ScanParams& p, int r, float la, int len, int j) {
  if (j >= len) return 0.f;
  const float k = static_cast<float>(len - 1 - j);
  const float dw = k * __expf(la * k);
  return p.kind[r] == kSlotStale ? -dw : dw;
}

// Index of state element (feature f, payload column c) of the boundary state
// arrays [B,H,R,Dk,Dv].
__device__ __forceinline__ size_t boundary_index(const ScanParams& p, int b, int h, int r, int f, int c) {
  return ((((static_cast<size_t>(b) * p.H + h) * p.R + r) * p.Dk + f) * p.Dv) + c;
}

// Intra-tile weights of every caller slot of head h at distances k =
// 0..kTile-1 into shared memory (`tab`: RU * kTile floats): exp(la_r k), or
// 1 - exp(la_r k) for a stale slot, so that w_r(i, j) = tab[r * kTile + i - j]
// for j <= i.  Visible after the next barrier.
__device__ __forceinline__ void fill_decay(const ScanParams& p, int h, float* tab) {
  for (int i = threadIdx.x; i < p.RU * kTile; i += blockDim.x) {
    const int r = i / kTile, k = i % kTile;
    const float x = head_la(p, r, h) * static_cast<float>(k);
    tab[i] = p.la[r] == nullptr ? 1.f : p.kind[r] == kSlotStale ? one_minus_exp(x) : __expf(x);
  }
}

// Thread mapping of the tile-prefix kernels.  A thread carries 8 consecutive
// features (f8*8 ..) of one value column c of one state through the tiles.
// Lanes 0-7 take 8 consecutive value columns and lanes 8 apart consecutive
// feature groups, so a warp touches whole 128-byte lines both in the f32
// states (value-major: 4 feature groups x 32 B per column) and in the bf16
// images (core-matrix order: 8 columns x 16 B per feature group).
// Grid: x = feature-group blocks of 32, y = R * (DvP / 8), z = B * H.
struct PrefixLane {
  int f8, c, r, b, h;
  bool active;
};
__device__ __forceinline__ PrefixLane prefix_lane(const ScanParams& p) {
  PrefixLane l;
  const int cblocks = p.DvP / 8;
  l.r = blockIdx.y / cblocks;
  l.c = (blockIdx.y % cblocks) * 8 + (threadIdx.x & 7);
  l.f8 = blockIdx.x * 32 + (threadIdx.x >> 3);
  l.b = blockIdx.z / p.H;
  l.h = blockIdx.z % p.H;
  l.active = l.f8 < p.DkM / 8;
  return l;
}
__host__ __device__ inline dim3 prefix_grid(int DkM, int DvP, int R, int BH) {
  return dim3((DkM / 8 + 31) / 32, R * (DvP / 8), BH);
}
constexpr int kPrefixBatch = 8;   // tiles whose states are loaded together
constexpr int kSegTiles = 16;     // tiles per segment of the two-level prefix

// Segments of the backward's two-level prefix: used for sequences of two or
// more segments without stale slots (whose paired lanes run the serial
// chain).
__host__ __device__ inline int prefix_segments(int NT, bool any_stale) {
  return (!any_stale && NT >= 2 * kSegTiles) ? (NT + kSegTiles - 1) / kSegTiles : 0;
}

// Lane of a two-level prefix kernel: as prefix_lane, with the segment in
// blockIdx.z (z = bh * NS + s) and blocks of min(256, DkM) threads.
struct SegLane {
  PrefixLane l;
  int s;
};
__device__ __forceinline__ SegLane seg_lane(const ScanParams& p) {
  SegLane o;
  const int cblocks = p.DvP / 8;
  const int per_block = blockDim.x >> 3;    // feature groups per block
  o.l.r = blockIdx.y / cblocks;
  o.l.c = (blockIdx.y % cblocks) * 8 + (threadIdx.x & 7);
  o.l.f8 = blockIdx.x * per_block + (threadIdx.x >> 3);
  const int bh = blockIdx.z / p.NS;
  o.s = blockIdx.z % p.NS;
  o.l.b = bh / p.H;
  o.l.h = bh % p.H;
  o.l.active = o.l.f8 < p.DkM / 8;
  return o;
}
__host__ __device__ inline int seg_threads(int DkM) { return DkM < 256 ? DkM : 256; }
__host__ __device__ inline dim3 seg_grid(int DkM, int DvP, int R, int BH, int NS) {
  const int per_block = seg_threads(DkM) / 8;
  return dim3((DkM / 8 + per_block - 1) / per_block, R * (DvP / 8), BH * NS);
}
__device__ __forceinline__ size_t seg_index(const ScanParams& p, int b, int h, int r, int s) {
  return (((static_cast<size_t>(b) * p.H + h) * p.R + r) * p.NS + s);
}

// The payload tile of a tile's rows: v, then the v_unit constant columns.
__device__ __forceinline__ void load_payload(const ScanParams& p, const Tile& t, const __nv_bfloat16* src, int rows) {
  load_tile(t, src, p.vs[2], rows, p.Dv - p.v_unit, p.v_unit ? p.Dv - p.v_unit : -1, p.v_unit);
}

__device__ __forceinline__ void store_out(void* base, bool bf16, size_t idx, float v) {
  if (bf16) {
    reinterpret_cast<__nv_bfloat16*>(base)[idx] = __float2bfloat16_rn(v);
  } else {
    reinterpret_cast<float*>(base)[idx] = v;
  }
}

// Build a tile whose row t is `scale(t) * row_t(src)` for a bf16 row-major
// source: a cooperative, coalesced copy (load_tile), then thread t rescales
// its own row in shared memory (conflict-free in the core-matrix layout).
// Rows >= rows_valid and columns >= cols_valid are zero; `unit_col` (if >= 0)
// is 1 before scaling.  Requires blockDim.x == kThreads and t.rows == kTile.
template <class Scale>
__device__ __forceinline__ void load_scaled_rows(const Tile& t, const __nv_bfloat16* __restrict__ src, long long ld,
                                                 int rows_valid, int cols_valid, int unit_col, Scale scale) {
  load_tile(t, src, ld, rows_valid, cols_valid, unit_col);
  cp_async_wait_all();
  __syncthreads();
  const int r = my_row();
  const float s = scale(r);
  for (int j = my_part(); j < t.cols / 8; j += kParts) {
    float f[8];
    unpack8(tile_ld16(t, r, j), f);
#pragma unroll
    for (int e = 0; e < 8; ++e) f[e] *= s;
    tile_st16(t, r, j, pack8(f));
  }
}

}  // namespace ts
