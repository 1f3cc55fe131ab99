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
// takes kRowsPerWarp of them, lanes striding the value columns in 8-byte
// pairs; rows of 64 or 128 columns are loaded a batch of rows at a time
// before any arithmetic (several rows' loads in flight per warp).
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

// Columns [c, c + V) of a row as floats (V = 2: one 8-byte load).
template <int V>
__device__ __forceinline__ void ld_cols(const float* __restrict__ src, float (&x)[V]) {
  if constexpr (V == 2) {
    const float2 v = __ldg(reinterpret_cast<const float2*>(src));
    x[0] = v.x;
    x[1] = v.y;
  } else {
    x[0] = __ldg(src);
  }
}

template <int V>
__device__ __forceinline__ void st_bf16_cols(__nv_bfloat16* dst, const float (&x)[V]) {
  if constexpr (V == 2) {
    *reinterpret_cast<__nv_bfloat162*>(dst) = __floats2bfloat162_rn(x[0], x[1]);
  } else {
    dst[0] = __float2bfloat16_rn(x[0]);
  }
}

// The slot count N = 1 + J is a template parameter so that the per-slot
// arrays stay in registers; each lane takes V adjacent value columns at a
// time (V = 2 when the row widths allow 8-byte loads).  With G > 0 the row
// width is exactly G groups of 32 V columns: a warp then issues the loads of
// a batch of rows before any arithmetic (the loads of different rows are
// independent), which keeps several rows' loads in flight per warp.  G = 0 is
// the general loop over column groups, one row at a time.
template <int N, int V, int G>
struct ReadBatch {
  // rows of one batch, bounded by the registers it holds
  static constexpr int kRegs = G > 0 ? N + G * V * (N + 1) : 1;
  static constexpr int kRows = G == 0 ? 1 : (64 / kRegs >= 8 ? 8 : 64 / kRegs >= 4 ? 4 : 64 / kRegs >= 2 ? 2 : 1);
};

template <int N, int V, int G>
__global__ void __launch_bounds__(kReadWarps * 32) kread_fwd_kernel(ReadParams p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y, b = blockIdx.z;
  float coef[5];
  slot_coefs(p, h, coef);
  const int width = p.d + p.mass_cols;
  const size_t bh = static_cast<size_t>(b) * p.H + h;
  const int tw = blockIdx.x * kReadRows + warp * kRowsPerWarp;
  if constexpr (G > 0) {
    constexpr int kB = ReadBatch<N, V, G>::kRows;
    for (int i0 = 0; i0 < kRowsPerWarp; i0 += kB) {
      float mass[kB][N], acc[kB][G][V], x[kB][N][G][V];
#pragma unroll
      for (int i = 0; i < kB; ++i) {
        const int t = tw + i0 + i;
        const size_t row = bh * p.T + (t < p.T ? t : 0);
#pragma unroll
        for (int s = 0; s < N; ++s) mass[i][s] = p.mass_cols ? __ldg(p.out[s] + row * width + p.d) : 0.f;
#pragma unroll
        for (int k = 0; k < G; ++k) {
          const int c = V * lane + 32 * V * k;
          ld_cols<V>(p.y0 + row * p.d + c, acc[i][k]);
#pragma unroll
          for (int s = 0; s < N; ++s) ld_cols<V>(p.out[s] + row * width + c, x[i][s][k]);
        }
      }
#pragma unroll
      for (int i = 0; i < kB; ++i) {
        const int t = tw + i0 + i;
        if (t >= p.T) break;
        __nv_bfloat16* yrow = p.y + ((static_cast<size_t>(b) * p.T + t) * p.H + h) * p.d;
#pragma unroll
        for (int s = 0; s < N; ++s) {
          const float scale = p.mass_cols ? coef[s] / (mass[i][s] + p.eps) : coef[s];
#pragma unroll
          for (int k = 0; k < G; ++k)
#pragma unroll
            for (int e = 0; e < V; ++e) acc[i][k][e] += scale * x[i][s][k][e];
        }
#pragma unroll
        for (int k = 0; k < G; ++k) st_bf16_cols<V>(yrow + V * lane + 32 * V * k, acc[i][k]);
      }
    }
  } else {
#pragma unroll 4
    for (int i = 0; i < kRowsPerWarp; ++i) {
      const int t = tw + i;
      if (t >= p.T) break;
      const size_t row = bh * p.T + t;  // [B, H, T] row index
      float scale[N];
#pragma unroll
      for (int s = 0; s < N; ++s)
        scale[s] = p.mass_cols ? coef[s] / (__ldg(p.out[s] + row * width + p.d) + p.eps) : coef[s];
      __nv_bfloat16* yrow = p.y + ((static_cast<size_t>(b) * p.T + t) * p.H + h) * p.d;
      for (int c = V * lane; c < p.d; c += 32 * V) {
        float acc[V], x[V];
        ld_cols<V>(p.y0 + row * p.d + c, acc);
#pragma unroll
        for (int s = 0; s < N; ++s) {
          ld_cols<V>(p.out[s] + row * width + c, x);
#pragma unroll
          for (int e = 0; e < V; ++e) acc[e] += scale[s] * x[e];
        }
        st_bf16_cols<V>(yrow + c, acc);
      }
    }
  }
}

// One row of the read backward for the columns this lane holds: dN rounded
// to bf16 (written), dy0 (written), and the lane's partial sums of
// dy . mem_s and of the rounded dN_s . mem_s.
template <int N, int V>
__device__ __forceinline__ void read_bwd_cols(const ReadParams& p, const float* coef, const float* inv, size_t row,
                                              int width, int c, const float (&dyc)[V], const float (&x)[N][V],
                                              float* exact, float* consistent) {
  if (p.dy0 != nullptr) {
    if constexpr (V == 2) {
      *reinterpret_cast<float2*>(p.dy0 + row * p.d + c) = make_float2(dyc[0], dyc[1]);
    } else {
      p.dy0[row * p.d + c] = dyc[0];
    }
  }
#pragma unroll
  for (int s = 0; s < N; ++s) {
    float dn[V];
#pragma unroll
    for (int e = 0; e < V; ++e) {
      // mass_cols == 0 (unnormalized read): mem_s = N_s and dN_s = c_s dy
      const float mem = x[s][e] * inv[s];
      dn[e] = p.mass_cols ? coef[s] * dyc[e] * inv[s] : coef[s] * dyc[e];
      exact[s] += dyc[e] * mem;
      // dN is rounded first; the mass gradient uses the rounded values
      consistent[s] += __bfloat162float(__float2bfloat16_rn(dn[e])) * mem;
    }
    st_bf16_cols<V>(p.dout[s] + row * width + c, dn);
  }
}

template <int V>
__device__ __forceinline__ void ld_dy(const ReadParams& p, size_t yidx, int c, float (&x)[V]) {
  if (p.dy_bf16) {
    const __nv_bfloat16* d = reinterpret_cast<const __nv_bfloat16*>(p.dy) + yidx + c;
    if constexpr (V == 2) {
      const float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(d));
      x[0] = v.x;
      x[1] = v.y;
    } else {
      x[0] = __bfloat162float(d[0]);
    }
  } else {
    ld_cols<V>(reinterpret_cast<const float*>(p.dy) + yidx + c, x);
  }
}

// Row totals of the backward from the lanes' partial sums: dy . mem_s into
// dymem, and the mass gradient dD_s = -sum dN_s mem_s written as bf16 hi (+ lo).
template <int N>
__device__ __forceinline__ void read_bwd_row_end(const ReadParams& p, size_t row, int width, int lane,
                                                 const float* exact, const float* consistent, float* dymem) {
#pragma unroll
  for (int s = 0; s < N; ++s) {
    dymem[s] = warp_sum(exact[s]);  // dy . mem_s
    if (p.mass_cols) {
      const float dD = -warp_sum(consistent[s]);
      if (lane == 0) {
        const __nv_bfloat16 hi = __float2bfloat16_rn(dD);
        p.dout[s][row * width + p.d] = hi;
        if (p.mass_cols == 2) p.dout[s][row * width + p.d + 1] = __float2bfloat16_rn(dD - __bfloat162float(hi));
      }
    }
  }
}

template <int N, int V, int G>
__global__ void __launch_bounds__(kReadWarps * 32) kread_bwd_kernel(ReadParams p) {
  __shared__ float red[kReadWarps][4];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y, b = blockIdx.z;
  float coef[5];
  slot_coefs(p, h, coef);
  const int width = p.d + p.mass_cols;
  const size_t bh = static_cast<size_t>(b) * p.H + h;
  const int tw = blockIdx.x * kReadRows + warp * kRowsPerWarp;
  float deta[4] = {0.f, 0.f, 0.f, 0.f};  // this warp's rows (every lane holds the sums)
  auto add_deta = [&](const float* dymem) {
    // fast: d eta_j = dy.mem(1+j) - dy.mem(0); stale: d eta_j = -dy.mem(1+j)
#pragma unroll
    for (int j = 0; j < N - 1; ++j) deta[j] += (p.mode == 1) ? dymem[1 + j] - dymem[0] : -dymem[1 + j];
  };
  if constexpr (G > 0) {
    // the backward keeps more per row (dN, the partial sums): a smaller batch
    // for three and more slots keeps its registers within two blocks per SM
    constexpr int kB = N >= 3 ? (ReadBatch<N, V, G>::kRows > 2 ? 2 : ReadBatch<N, V, G>::kRows) : ReadBatch<N, V, G>::kRows;
    for (int i0 = 0; i0 < kRowsPerWarp; i0 += kB) {
      float mass[kB][N], dy[kB][G][V], x[kB][G][N][V];
#pragma unroll
      for (int i = 0; i < kB; ++i) {
        const int t = tw + i0 + i;
        const int tt = t < p.T ? t : 0;
        const size_t row = bh * p.T + tt;
        const size_t yidx = ((static_cast<size_t>(b) * p.T + tt) * p.H + h) * p.d;
#pragma unroll
        for (int s = 0; s < N; ++s) mass[i][s] = p.mass_cols ? __ldg(p.out[s] + row * width + p.d) : 0.f;
#pragma unroll
        for (int k = 0; k < G; ++k) {
          const int c = V * lane + 32 * V * k;
          ld_dy<V>(p, yidx, c, dy[i][k]);
#pragma unroll
          for (int s = 0; s < N; ++s) ld_cols<V>(p.out[s] + row * width + c, x[i][k][s]);
        }
      }
#pragma unroll
      for (int i = 0; i < kB; ++i) {
        const int t = tw + i0 + i;
        if (t >= p.T) break;
        const size_t row = bh * p.T + t;
        float inv[N], exact[N], consistent[N], dymem[N];
#pragma unroll
        for (int s = 0; s < N; ++s) {
          inv[s] = p.mass_cols ? 1.f / (mass[i][s] + p.eps) : 1.f;
          exact[s] = consistent[s] = 0.f;
        }
#pragma unroll
        for (int k = 0; k < G; ++k)
          read_bwd_cols<N, V>(p, coef, inv, row, width, V * lane + 32 * V * k, dy[i][k], x[i][k], exact,
                              consistent);
        read_bwd_row_end<N>(p, row, width, lane, exact, consistent, dymem);
        add_deta(dymem);
      }
    }
  } else {
#pragma unroll 2
    for (int i = 0; i < kRowsPerWarp; ++i) {
      const int t = tw + i;
      if (t >= p.T) break;
      const size_t row = bh * p.T + t;
      const size_t yidx = ((static_cast<size_t>(b) * p.T + t) * p.H + h) * p.d;
      float inv[N], exact[N], consistent[N], dymem[N];
#pragma unroll
      for (int s = 0; s < N; ++s) {
        inv[s] = p.mass_cols ? 1.f / (__ldg(p.out[s] + row * width + p.d) + p.eps) : 1.f;
        exact[s] = consistent[s] = 0.f;
      }
      for (int c = V * lane; c < p.d; c += 32 * V) {
        float dyc[V], x[N][V];
        ld_dy<V>(p, yidx, c, dyc);
#pragma unroll
        for (int s = 0; s < N; ++s) ld_cols<V>(p.out[s] + row * width + c, x[s]);
        read_bwd_cols<N, V>(p, coef, inv, row, width, c, dyc, x, exact, consistent);
      }
      read_bwd_row_end<N>(p, row, width, lane, exact, consistent, dymem);
      add_deta(dymem);
    }
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

template <int N, int V, int G>
static int launch_kread_g(const ReadParams& p, cudaStream_t s, bool backward) {
  const dim3 grid(ceil_div(p.T, kReadRows), p.H, p.B);
  if (backward) {
    kread_bwd_kernel<N, V, G><<<grid, kReadWarps * 32, 0, s>>>(p);
    return check_launch("kread_bwd_kernel");
  }
  kread_fwd_kernel<N, V, G><<<grid, kReadWarps * 32, 0, s>>>(p);
  return check_launch("kread_fwd_kernel");
}

template <int N>
static int launch_kread_n(const ReadParams& p, cudaStream_t s, bool backward) {
  // 8-byte column pairs where every row start stays 8-byte aligned; whole
  // groups of 64 columns (one or two) take the batched loads
  const bool pairs = (p.d % 2) == 0 && ((p.d + p.mass_cols) % 2) == 0;
  if (pairs && p.d == 64) return launch_kread_g<N, 2, 1>(p, s, backward);
  if (pairs && p.d == 128) return launch_kread_g<N, 2, 2>(p, s, backward);
  if (pairs) return launch_kread_g<N, 2, 0>(p, s, backward);
  return launch_kread_g<N, 1, 0>(p, s, backward);
}

static int launch_kread(const ReadParams& p, cudaStream_t s, bool backward) {
  switch (1 + p.J) {
    case 1: return launch_kread_n<1>(p, s, backward);
    case 2: return launch_kread_n<2>(p, s, backward);
    case 3: return launch_kread_n<3>(p, s, backward);
    case 4: return launch_kread_n<4>(p, s, backward);
    default: return launch_kread_n<5>(p, s, backward);
  }
}

int launch_kread_fwd(const ReadParams& p, cudaStream_t s) { return launch_kread(p, s, false); }

int launch_kread_bwd(const ReadParams& p, cudaStream_t s) { return launch_kread(p, s, true); }

}  // namespace ts
