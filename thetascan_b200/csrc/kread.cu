// Key-mass normalized read and temporal-view blend of the kernel family
// (also the unnormalized blend, mass_cols = 0: mem(s) = N_s, for the
// unnormalized and feature-mass reads, engine.py:402-416, 443-456).
//
// The scans deliver, per retention slot s, the augmented read
// out_s = [N_s | D_s] (numerator and score mass, reference engine.py:430-442),
// with the mass column once or twice (`mass_cols`).  Every view is one slot
// (interface.py:251-307) and the mixer blends views (block.py:676-718):
//   mode 0  plain sum          y = y0 + mem(0)
//   mode 1  bank, fast         y = y0 + (1 - sum_j eta_j) mem(0) + sum_j eta_j mem(1+j)
//   mode 2  bank, stale        y = y0 + mem(0) - sum_j eta_j mem(1+j)
// with mem(s) = N_s / (D_s + eps) and y0 = q + W2 phi(q).  In mode 2 slot 1+j
// is the stale scan of branch j (weights 1 - alpha_j^(t-i), the view
// S_sum - S_fast of interface.py:251-279, formed inside the scan), and the
// zero-memory base read that the stale blend subtracts is y0 itself.
//
// Backward: with c_s the slot's coefficient, dN_s = c_s dy / (D_s + eps) is
// rounded to bf16 FIRST and the mass gradient is formed from the rounded
// values, dD_s = -sum_c dN_s[c] mem_s[c], in f32.  The scan backward sees
// dout . [v | 1] = dN . (v - mem) for every key: the cancellation of the
// quotient rule happens inside its f32 sums instead of between two separately
// rounded numbers (whose residual grows like 1/D for small masses).  With two
// mass columns dD travels as bf16 hi + lo, exact to ~2^-17.
// A block owns kReadRows consecutive tokens of one (batch, head); each warp
// takes kRowsPerWarp of them, lanes striding the value columns, with
// read-only loads the compiler may batch across rows.
#include "capi_internal.h"
#include "common.cuh"

namespace ts {

struct ReadParams {
  int B, H, T, d;
  int J;                       // recency branches (slots 1..J)
  int mode;                    // 0 sum, 1 fast, 2 stale
  int mass_cols;               // mass columns after the d value columns (1 or 2; 0: unnormalized read)
  float eps;
  const float* out[5];         // slot outputs [B, H, T, d + mass_cols] f32
  const float* eta;            // [J, H] f32
  const float* y0;             // [B, H, T, d] f32
  __nv_bfloat16* y;            // [B, T, H, d]
  // backward
  const void* dy;              // [B, T, H, d]
  int dy_bf16;
  __nv_bfloat16* dout[5];      // [B, H, T, d + mass_cols]
  float* dy0;                  // [B, H, T, d] or null
  float* deta;                 // [J, H] (accumulated)
};

namespace {

// Output coefficient of every slot (one view per slot).
__device__ __forceinline__ void slot_coefs(const ReadParams& p, int h, float* coef) {
  float eta_sum = 0.f;
  for (int j = 0; j < p.J; ++j) eta_sum += __ldg(p.eta + j * p.H + h);
  coef[0] = (p.mode == 1) ? 1.f - eta_sum : 1.f;
  for (int j = 0; j < p.J; ++j) {
    const float eta = __ldg(p.eta + j * p.H + h);
    coef[1 + j] = (p.mode == 1) ? eta : -eta;
  }
}

__device__ __forceinline__ float slot_val(const ReadParams& p, int s, size_t row, int c) {
  return __ldg(p.out[s] + row * (p.d + p.mass_cols) + c);
}

constexpr int kReadWarps = 8;
constexpr int kRowsPerWarp = 8;
constexpr int kReadRows = kReadWarps * kRowsPerWarp;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

}  // namespace

__global__ void __launch_bounds__(kReadWarps * 32) kread_fwd_kernel(ReadParams p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y, b = blockIdx.z;
  float coef[5];
  slot_coefs(p, h, coef);
  const int n = 1 + p.J;
  const size_t bh = static_cast<size_t>(b) * p.H + h;
#pragma unroll 4
  for (int i = 0; i < kRowsPerWarp; ++i) {
    const int t = blockIdx.x * kReadRows + warp * kRowsPerWarp + i;
    if (t >= p.T) break;
    const size_t row = bh * p.T + t;  // [B, H, T] row index
    float scale[5];
    for (int s = 0; s < n; ++s) scale[s] = p.mass_cols ? coef[s] / (slot_val(p, s, row, p.d) + p.eps) : coef[s];
    __nv_bfloat16* yrow = p.y + ((static_cast<size_t>(b) * p.T + t) * p.H + h) * p.d;
    for (int c = lane; c < p.d; c += 32) {
      float acc = __ldg(p.y0 + row * p.d + c);
      for (int s = 0; s < n; ++s) acc += scale[s] * slot_val(p, s, row, c);
      yrow[c] = __float2bfloat16_rn(acc);
    }
  }
}

__global__ void __launch_bounds__(kReadWarps * 32) kread_bwd_kernel(ReadParams p) {
  __shared__ float red[kReadWarps][4];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y, b = blockIdx.z;
  float coef[5];
  slot_coefs(p, h, coef);
  const int n = 1 + p.J;
  const int width = p.d + p.mass_cols;
  const size_t bh = static_cast<size_t>(b) * p.H + h;
  float deta[4] = {0.f, 0.f, 0.f, 0.f};  // this warp's rows (every lane holds the sums)
#pragma unroll 2
  for (int i = 0; i < kRowsPerWarp; ++i) {
    const int t = blockIdx.x * kReadRows + warp * kRowsPerWarp + i;
    if (t >= p.T) break;
    const size_t row = bh * p.T + t;
    const size_t yidx = ((static_cast<size_t>(b) * p.T + t) * p.H + h) * p.d;
    auto dy_at = [&](int c) {
      return p.dy_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.dy)[yidx + c])
                       : reinterpret_cast<const float*>(p.dy)[yidx + c];
    };
    float dymem[5];
    for (int s = 0; s < n; ++s) {
      if (p.mass_cols == 0) {
        // unnormalized read: mem_s = N_s
        float dot = 0.f;
        for (int c = lane; c < p.d; c += 32) {
          const float dyc = dy_at(c);
          p.dout[s][row * width + c] = __float2bfloat16_rn(coef[s] * dyc);
          dot += dyc * slot_val(p, s, row, c);
        }
        dymem[s] = warp_sum(dot);
        continue;
      }
      const float inv = 1.f / (slot_val(p, s, row, p.d) + p.eps);
      float exact = 0.f, consistent = 0.f;
      for (int c = lane; c < p.d; c += 32) {
        const float dyc = dy_at(c);
        const float mem = slot_val(p, s, row, c) * inv;
        const __nv_bfloat16 dn = __float2bfloat16_rn(coef[s] * dyc * inv);
        p.dout[s][row * width + c] = dn;
        exact += dyc * mem;
        consistent += __bfloat162float(dn) * mem;
      }
      dymem[s] = warp_sum(exact);           // dy . mem_s
      const float dD = -warp_sum(consistent);
      if (lane == 0) {
        const __nv_bfloat16 hi = __float2bfloat16_rn(dD);
        p.dout[s][row * width + p.d] = hi;
        if (p.mass_cols == 2) p.dout[s][row * width + p.d + 1] = __float2bfloat16_rn(dD - __bfloat162float(hi));
      }
    }
    if (p.dy0 != nullptr)
      for (int c = lane; c < p.d; c += 32) p.dy0[row * p.d + c] = dy_at(c);
    // fast: d eta_j = dy.mem(1+j) - dy.mem(0); stale: d eta_j = -dy.mem(1+j)
    for (int j = 0; j < p.J; ++j) deta[j] += (p.mode == 1) ? dymem[1 + j] - dymem[0] : -dymem[1 + j];
  }
  if (p.deta == nullptr || p.J == 0) return;  // uniform across the block
  if (lane == 0)
    for (int j = 0; j < 4; ++j) red[warp][j] = deta[j];
  __syncthreads();
  if (threadIdx.x < p.J) {
    float sum = 0.f;
    for (int w = 0; w < kReadWarps; ++w) sum += red[w][threadIdx.x];
    atomicAdd(p.deta + threadIdx.x * p.H + h, sum);
  }
}

int launch_kread_fwd(const ReadParams& p, cudaStream_t s) {
  kread_fwd_kernel<<<dim3(ceil_div(p.T, kReadRows), p.H, p.B), kReadWarps * 32, 0, s>>>(p);
  return check_launch("kread_fwd_kernel");
}

int launch_kread_bwd(const ReadParams& p, cudaStream_t s) {
  kread_bwd_kernel<<<dim3(ceil_div(p.T, kReadRows), p.H, p.B), kReadWarps * 32, 0, s>>>(p);
  return check_launch("kread_bwd_kernel");
}

}  // namespace ts
