// Float32 streams of the multi-view scan (ts_scan_args.f32_streams): shared
// between the C-ABI layer and the CUDA-core kernels of scan_f32.cu.
#pragma once

#include "capi_internal.h"

namespace ts {

constexpr int kF32MaxDk = 256;
constexpr int kF32MaxDv = 256;

struct ScanF32Params {
  int B, H, T, Dk, Dv;
  int TL;                     // tile length in tokens (64, or 32 when 64 exceeds shared memory)
  int NT, R, v_unit;          // tiles, retentions, constant 1 columns after v
  const float* q;
  const float* k;
  const float* v;
  long long qs[3], ks[3], vs[3];
  const float* la[TS_MAX_RETENTIONS];  // [H] or null (plain sum)
  const float* las[TS_MAX_RETENTIONS]; // [B,H,T] per-token log-retention stream, or null
  float* closing;                      // [B*H][NT][R] exp(sum of a tile's stream), stream retentions
  float* out[TS_MAX_RETENTIONS];       // [B,H,T,Dv]
  // [B*H][NT][R][Dk][Dv]: each tile's local update, then (after the tile
  // prefix) the state entering each tile
  float* states;
  // backward
  const float* dout[TS_MAX_RETENTIONS];  // [B,H,T,Dv]
  float* dq;                             // [B,H,T,Dk]
  float* dk;
  float* dv;                             // [B,H,T,Dv]
  float* dla[TS_MAX_RETENTIONS];         // [H], accumulated; null = not wanted
  float* dlas[TS_MAX_RETENTIONS];        // [B,H,T] gradient of a stream (written); null = not wanted
  float* zterm;                          // [B*H][NT][R] C_n <G(n), S_in(n)> of stream retentions (zeroed)
  // [B*H][NT][R][Dk][Dv]: each tile's local read gradient, then the gradient
  // of the state leaving each tile
  float* gstates;
};

size_t scan_f32_smem(int TL, int Dk, int Dv, bool backward);
int launch_scan_f32_fwd(const ScanF32Params& p, cudaStream_t s);
int launch_scan_f32_bwd(const ScanF32Params& p, cudaStream_t s);

}  // namespace ts
