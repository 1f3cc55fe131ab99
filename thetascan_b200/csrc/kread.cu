// Key-mass normalized read and temporal-view blend of the kernel family.
//
// The scans deliver, per retention slot s, the augmented read
// out_s = [N_s | D_s] (numerator and score mass, reference engine.py:430-442).
// Views combine slots (interface.py:251-307) and the mixer blends views
// (block.py:676-718):
//   mode 0  plain sum          y = y0 + mem(slot 0)
//   mode 1  bank, fast         y = y0 + (1 - sum_j eta_j) mem(0) + sum_j eta_j mem(1+j)
//   mode 2  bank, stale        y = y0 + mem(0) - sum_j eta_j mem(slot 0 - slot 1+j)
// with mem(view) = N_view / (D_view + eps) and y0 = q + W2 phi(q).
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
  float eps;
  const float* out[5];         // slot outputs [B, H, T, d+1] f32
  const float* eta;            // [J, H] f32
  const float* y0;             // [B, H, T, d] f32
  __nv_bfloat16* y;            // [B, T, H, d]
  // backward
  const void* dy;              // [B, T, H, d]
  int dy_bf16;
  __nv_bfloat16* dout[5];      // [B, H, T, d+1]
  float* dy0;                  // [B, H, T, d] or null
  float* deta;                 // [J, H] (accumulated)
};

namespace {

struct ViewSet {
  int n;                 // number of views
  float coef[5];         // output coefficient of each view
  int slot_a[5], slot_b[5];  // view = slot_a - slot_b (slot_b < 0: none)
};

__device__ __forceinline__ ViewSet make_views(const ReadParams& p, int h) {
  ViewSet v;
  v.n = 1 + p.J;
  float eta_sum = 0.f;
  for (int j = 0; j < p.J; ++j) eta_sum += __ldg(p.eta + j * p.H + h);
  v.slot_a[0] = 0;
  v.slot_b[0] = -1;
  v.coef[0] = (p.mode == 1) ? 1.f - eta_sum : 1.f;
  for (int j = 0; j < p.J; ++j) {
    const float eta = __ldg(p.eta + j * p.H + h);
    if (p.mode == 1) {
      v.slot_a[1 + j] = 1 + j;
      v.slot_b[1 + j] = -1;
      v.coef[1 + j] = eta;
    } else {
      v.slot_a[1 + j] = 0;
      v.slot_b[1 + j] = 1 + j;
      v.coef[1 + j] = -eta;
    }
  }
  return v;
}

__device__ __forceinline__ float slot_val(const ReadParams& p, int s, size_t row, int c) {
  return __ldg(p.out[s] + row * (p.d + 1) + c);
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
  const ViewSet vs = make_views(p, h);
  const size_t bh = static_cast<size_t>(b) * p.H + h;
#pragma unroll 4
  for (int i = 0; i < kRowsPerWarp; ++i) {
    const int t = blockIdx.x * kReadRows + warp * kRowsPerWarp + i;
    if (t >= p.T) break;
    const size_t row = bh * p.T + t;  // [B, H, T] row index
    float inv_den[5];
    for (int k = 0; k < vs.n; ++k) {
      float D = slot_val(p, vs.slot_a[k], row, p.d);
      if (vs.slot_b[k] >= 0) D -= slot_val(p, vs.slot_b[k], row, p.d);
      inv_den[k] = 1.f / (D + p.eps);
    }
    __nv_bfloat16* yrow = p.y + ((static_cast<size_t>(b) * p.T + t) * p.H + h) * p.d;
    for (int c = lane; c < p.d; c += 32) {
      float acc = __ldg(p.y0 + row * p.d + c);
      for (int k = 0; k < vs.n; ++k) {
        float N = slot_val(p, vs.slot_a[k], row, c);
        if (vs.slot_b[k] >= 0) N -= slot_val(p, vs.slot_b[k], row, c);
        acc += vs.coef[k] * N * inv_den[k];
      }
      yrow[c] = __float2bfloat16_rn(acc);
    }
  }
}

__global__ void __launch_bounds__(kReadWarps * 32) kread_bwd_kernel(ReadParams p) {
  __shared__ float red[kReadWarps][4];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y, b = blockIdx.z;
  const ViewSet vs = make_views(p, h);
  const size_t bh = static_cast<size_t>(b) * p.H + h;
  const int nslots = 1 + p.J;
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
    float inv_den[5], dymem[5];
    for (int k = 0; k < vs.n; ++k) {
      float D = slot_val(p, vs.slot_a[k], row, p.d);
      if (vs.slot_b[k] >= 0) D -= slot_val(p, vs.slot_b[k], row, p.d);
      inv_den[k] = 1.f / (D + p.eps);
      float s = 0.f;
      for (int c = lane; c < p.d; c += 32) {
        float N = slot_val(p, vs.slot_a[k], row, c);
        if (vs.slot_b[k] >= 0) N -= slot_val(p, vs.slot_b[k], row, c);
        s += dy_at(c) * N;
      }
      dymem[k] = warp_sum(s) * inv_den[k];  // dy . mem_k
    }
    for (int c = lane; c <= p.d; c += 32) {
      float g[5] = {0.f, 0.f, 0.f, 0.f, 0.f};
      const float dyc = c < p.d ? dy_at(c) : 0.f;
      for (int k = 0; k < vs.n; ++k) {
        // d N_k = c_k dy / (D_k + eps);  d D_k = -c_k (dy . mem_k) / (D_k + eps)
        const float val = (c < p.d) ? vs.coef[k] * dyc * inv_den[k] : -vs.coef[k] * dymem[k] * inv_den[k];
        g[vs.slot_a[k]] += val;
        if (vs.slot_b[k] >= 0) g[vs.slot_b[k]] -= val;
      }
      for (int s = 0; s < nslots; ++s) p.dout[s][row * (p.d + 1) + c] = __float2bfloat16_rn(g[s]);
      if (c < p.d && p.dy0 != nullptr) p.dy0[row * p.d + c] = dyc;
    }
    // fast: d eta_j = dy.mem(1+j) - dy.mem(0); stale: d eta_j = -dy.mem(stale_j)
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
