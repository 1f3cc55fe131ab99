// Per-token maps of the Gauss--Newton fast-weight family (ts_b200_gn_rows).
//
// The GN write (src/thetascan/_core/ops/engine.py:161-340 of the reference,
// depth 1, one Jacobian step) and the two stages of its read
// (engine.py:455-528) are, per token and head, a handful of 128x128 per-head
// linear maps -- cuBLAS GEMMs over all tokens of a head -- joined by
// nonlinear row maps: an RMS normalisation, the activation and its first two
// derivatives, the damped diagonal solve, the mass normalisations of the
// reads.  This file holds those row maps, forward and backward, as one
// kernel per stage: a warp owns a row (lane l holds columns l, l+32, ...),
// row sums are warp shuffles, and a CTA walks a run of rows of one (batch,
// head) so that the threshold gradient folds into one atomic per column and
// CTA.  Every stage reads and writes its rows once; the stages are HBM-bound.
//
// Row maps (rows of [B,H,T,*] f32; W1 [H,m,d], W2 [H,d,m] applied outside):
//   write:  a = W1 k; inv = (mean a^2 + eps)^-1/2; p = a inv - tau;
//           h = sigma(p); s = sigma'(p) inv;               (WRITE_PRE)
//           O = W2 h; RS = (W2 o W2) s^2;
//           lam = (v - k - O) / (|h|^2 + |k|^2 RS + eps);  (WRITE_LAM)
//           U = W2^T lam; g = sigma'(p) U inv              (WRITE_G)
//   read:   a_q = W1 q; h0 = relu2(a_q inv_q - tau)        (QUERY_PRE)
//           pre = a_q + R[:m] / (R[m] + eps)  (R the stage-1 read, or R
//           unnormalised, or absent); hq = sigma(rms(pre) - tau)  (FEATURES)
//           y = q + W2 hq + C[:d] / (C[d] + eps)           (OUT)
#include "capi_internal.h"

namespace ts {

constexpr int kGnThreads = 256;          // 8 warps, one row each at a time
constexpr int kGnRowsPerCta = 64;
constexpr int kGnMaxWidth = 256;

struct GnRowParams {
  int B, H, T, d, m;
  int nonlin, flags;
  float eps;
  const float* tau;
  float* dtau;
  const float* in[8];
  float* out[4];
  __nv_bfloat16* out_bf16;  // bf16 copy of out[0] (forward stages), or null
};

// sigma, sigma', sigma'' of the fast net's nonlinearity
// (src/thetascan/_core/ops/nonlin.py of the reference: relu2, silu, tanh).
template <int NL>
struct Act;
template <>
struct Act<TS_GN_RELU2> {
  static __device__ __forceinline__ void eval(float x, float& f, float& d1, float& d2) {
    const float r = fmaxf(x, 0.f);
    f = r * r;
    d1 = 2.f * r;
    d2 = x > 0.f ? 2.f : 0.f;
  }
};
template <>
struct Act<TS_GN_SILU> {
  static __device__ __forceinline__ void eval(float x, float& f, float& d1, float& d2) {
    const float s = 1.f / (1.f + expf(-x));
    f = x * s;
    d1 = s * (1.f + x * (1.f - s));
    d2 = s * (1.f - s) * (2.f + x * (1.f - 2.f * s));
  }
};
template <>
struct Act<TS_GN_TANH> {
  static __device__ __forceinline__ void eval(float x, float& f, float& d1, float& d2) {
    const float t = tanhf(x);
    f = t;
    d1 = 1.f - t * t;
    d2 = -2.f * t * d1;
  }
};

__device__ __forceinline__ float gn_warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// lane's slots of a row: column c = lane + 32 i, zero beyond n
template <int W>
__device__ __forceinline__ void gn_load(float (&r)[W], const float* p, int n) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int i = 0; i < W; ++i) {
    const int c = lane + 32 * i;
    r[i] = c < n ? __ldg(p + c) : 0.f;
  }
}

template <int W>
__device__ __forceinline__ void gn_store(float* p, const float (&r)[W], int n) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int i = 0; i < W; ++i) {
    const int c = lane + 32 * i;
    if (c < n) p[c] = r[i];
  }
}

// out[0] of a forward stage: f32 and/or its bf16 copy (the scans' operand)
template <int W>
__device__ __forceinline__ void gn_store_out0(const GnRowParams& p, size_t off, const float (&r)[W], int n) {
  if (p.out[0]) gn_store<W>(p.out[0] + off, r, n);
  if (p.out_bf16) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int i = 0; i < W; ++i) {
      const int c = lane + 32 * i;
      if (c < n) p.out_bf16[off + c] = __float2bfloat16_rn(r[i]);
    }
  }
}

template <int W>
__device__ __forceinline__ void gn_store_acc(float* p, const float (&r)[W], int n, bool acc) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int i = 0; i < W; ++i) {
    const int c = lane + 32 * i;
    if (c < n) p[c] = acc ? p[c] + r[i] : r[i];
  }
}

// 1 / sqrt(mean(a^2) + eps) over the row's n columns
template <int W>
__device__ __forceinline__ float gn_inv_rms(const float (&a)[W], int n, float eps) {
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < W; ++i) s = fmaf(a[i], a[i], s);
  return 1.f / sqrtf(gn_warp_sum(s) / static_cast<float>(n) + eps);
}

// Adds the lanes' threshold-gradient slots of all warps of the CTA into
// dtau[h] (one atomic per column and CTA).
template <int W>
__device__ void gn_flush_dtau(const GnRowParams& p, const float (&acc)[W], int h) {
  __shared__ float part[kGnThreads / 32][kGnMaxWidth];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int i = 0; i < W; ++i) part[warp][lane + 32 * i] = acc[i];
  __syncthreads();
  for (int c = threadIdx.x; c < p.m; c += kGnThreads) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kGnThreads / 32; ++w) s += part[w][c];
    if (s != 0.f) atomicAdd(p.dtau + static_cast<size_t>(h) * p.m + c, s);
  }
}

// Rows of this CTA: a run of one (batch, head) row block.
struct GnRows {
  int bh, h, t0, t1;
  __device__ GnRows(const GnRowParams& p) {
    bh = blockIdx.y;
    h = bh % p.H;
    t0 = blockIdx.x * kGnRowsPerCta;
    t1 = min(p.T, t0 + kGnRowsPerCta);
  }
};

__device__ __forceinline__ size_t gn_row(const GnRowParams& p, int bh, int t) {
  return static_cast<size_t>(bh) * p.T + t;
}

template <int W>
__device__ __forceinline__ void gn_tau(float (&tau)[W], const GnRowParams& p, int h) {
  if (p.tau) gn_load<W>(tau, p.tau + static_cast<size_t>(h) * p.m, p.m);
  else
#pragma unroll
    for (int i = 0; i < W; ++i) tau[i] = 0.f;
}

// ---------------------------------------------------------------- forward

// in {a [m], k [d]} -> out {h [m], s2 [m], hh [1], kk [1]}
template <int NL, int W>
__global__ void __launch_bounds__(kGnThreads) gn_write_pre_kernel(GnRowParams p) {
  const GnRows rs(p);
  float tau[W];
  gn_tau<W>(tau, p, rs.h);
  for (int t = rs.t0 + (threadIdx.x >> 5); t < rs.t1; t += kGnThreads / 32) {
    const size_t r = gn_row(p, rs.bh, t);
    float a[W], k[W], h[W], s2[W];
    gn_load<W>(a, p.in[0] + r * p.m, p.m);
    gn_load<W>(k, p.in[1] + r * p.d, p.d);
    const float inv = gn_inv_rms<W>(a, p.m, p.eps);
    float hh = 0.f, kk = 0.f;
#pragma unroll
    for (int i = 0; i < W; ++i) {
      float f, d1, d2;
      Act<NL>::eval(fmaf(a[i], inv, -tau[i]), f, d1, d2);
      const bool in = (threadIdx.x & 31) + 32 * i < p.m;
      h[i] = in ? f : 0.f;
      const float s = d1 * inv;
      s2[i] = in ? s * s : 0.f;
      hh = fmaf(h[i], h[i], hh);
      kk = fmaf(k[i], k[i], kk);
    }
    hh = gn_warp_sum(hh);
    kk = gn_warp_sum(kk);
    gn_store_out0<W>(p, r * p.m, h, p.m);
    gn_store<W>(p.out[1] + r * p.m, s2, p.m);
    if ((threadIdx.x & 31) == 0) {
      p.out[2][r] = hh;
      p.out[3][r] = kk;
    }
  }
}

// in {v, k, O, RS [d], hh, kk [1]} -> out {lam [d]}
template <int W>
__global__ void __launch_bounds__(kGnThreads) gn_write_lam_kernel(GnRowParams p) {
  const GnRows rs(p);
  for (int t = rs.t0 + (threadIdx.x >> 5); t < rs.t1; t += kGnThreads / 32) {
    const size_t r = gn_row(p, rs.bh, t);
    float v[W], k[W], o[W], q[W], lam[W];
    gn_load<W>(v, p.in[0] + r * p.d, p.d);
    gn_load<W>(k, p.in[1] + r * p.d, p.d);
    gn_load<W>(o, p.in[2] + r * p.d, p.d);
    gn_load<W>(q, p.in[3] + r * p.d, p.d);
    const float hh = __ldg(p.in[4] + r), kk = __ldg(p.in[5] + r);
#pragma unroll
    for (int i = 0; i < W; ++i) lam[i] = (v[i] - k[i] - o[i]) / (fmaf(kk, q[i], hh) + p.eps);
    gn_store_out0<W>(p, r * p.d, lam, p.d);
  }
}

// in {a [m], U [m]} -> out {g [m]}
template <int NL, int W>
__global__ void __launch_bounds__(kGnThreads) gn_write_g_kernel(GnRowParams p) {
  const GnRows rs(p);
  float tau[W];
  gn_tau<W>(tau, p, rs.h);
  for (int t = rs.t0 + (threadIdx.x >> 5); t < rs.t1; t += kGnThreads / 32) {
    const size_t r = gn_row(p, rs.bh, t);
    float a[W], u[W], g[W];
    gn_load<W>(a, p.in[0] + r * p.m, p.m);
    gn_load<W>(u, p.in[1] + r * p.m, p.m);
    const float inv = gn_inv_rms<W>(a, p.m, p.eps);
#pragma unroll
    for (int i = 0; i < W; ++i) {
      float f, d1, d2;
      Act<NL>::eval(fmaf(a[i], inv, -tau[i]), f, d1, d2);
      g[i] = d1 * u[i] * inv;
    }
    gn_store_out0<W>(p, r * p.m, g, p.m);
  }
}

// in {a_q [m]} -> out {h0 [m]}: the positive slow features relu2(rms(a_q) - tau)
template <int W>
__global__ void __launch_bounds__(kGnThreads) gn_query_pre_kernel(GnRowParams p) {
  const GnRows rs(p);
  float tau[W];
  gn_tau<W>(tau, p, rs.h);
  for (int t = rs.t0 + (threadIdx.x >> 5); t < rs.t1; t += kGnThreads / 32) {
    const size_t r = gn_row(p, rs.bh, t);
    float a[W], h[W];
    gn_load<W>(a, p.in[0] + r * p.m, p.m);
    const float inv = gn_inv_rms<W>(a, p.m, p.eps);
#pragma unroll
    for (int i = 0; i < W; ++i) {
      const float x = fmaxf(fmaf(a[i], inv, -tau[i]), 0.f);
      h[i] = x * x;
    }
    gn_store_out0<W>(p, r * p.m, h, p.m);
  }
}

// The corrected preactivation of a read stage: a_q plus the stage-1 read R
// (flags bit 0: R has m + 1 columns, the last its mass; divide by mass + eps)
template <int W>
__device__ __forceinline__ float gn_pre(float (&pre)[W], float (&rd)[W], float& mass, const GnRowParams& p,
                                        size_t r) {
  gn_load<W>(pre, p.in[0] + r * p.m, p.m);
  mass = 0.f;
  if (!p.in[1]) {
#pragma unroll
    for (int i = 0; i < W; ++i) rd[i] = 0.f;
    return 1.f;
  }
  const bool norm = p.flags & 1;
  const int ld = norm ? p.m + 1 : p.m;
  gn_load<W>(rd, p.in[1] + r * ld, p.m);
  float scale = 1.f;
  if (norm) {
    mass = __ldg(p.in[1] + r * ld + p.m);
    scale = 1.f / (mass + p.eps);
  }
#pragma unroll
  for (int i = 0; i < W; ++i) pre[i] = fmaf(rd[i], scale, pre[i]);
  return scale;
}

// in {a_q [m], R [m(+1)] or NULL} -> out {hq [m]}
template <int NL, int W>
__global__ void __launch_bounds__(kGnThreads) gn_features_kernel(GnRowParams p) {
  const GnRows rs(p);
  float tau[W];
  gn_tau<W>(tau, p, rs.h);
  for (int t = rs.t0 + (threadIdx.x >> 5); t < rs.t1; t += kGnThreads / 32) {
    const size_t r = gn_row(p, rs.bh, t);
    float pre[W], rd[W], hq[W], mass;
    gn_pre<W>(pre, rd, mass, p, r);
    const float inv = gn_inv_rms<W>(pre, p.m, p.eps);
#pragma unroll
    for (int i = 0; i < W; ++i) {
      float f, d1, d2;
      Act<NL>::eval(fmaf(pre[i], inv, -tau[i]), f, d1, d2);
      hq[i] = f;
    }
    gn_store_out0<W>(p, r * p.m, hq, p.m);
  }
}

// in {q, base [d], C [d(+1)]} -> out {y [d]} (flags bit 0: C normalised by its mass column)
template <int W>
__global__ void __launch_bounds__(kGnThreads) gn_out_kernel(GnRowParams p) {
  const GnRows rs(p);
  const bool norm = p.flags & 1;
  const int ld = norm ? p.d + 1 : p.d;
  for (int t = rs.t0 + (threadIdx.x >> 5); t < rs.t1; t += kGnThreads / 32) {
    const size_t r = gn_row(p, rs.bh, t);
    float q[W], b[W], c[W], y[W];
    gn_load<W>(q, p.in[0] + r * p.d, p.d);
    gn_load<W>(b, p.in[1] + r * p.d, p.d);
    gn_load<W>(c, p.in[2] + r * ld, p.d);
    const float scale = norm ? 1.f / (__ldg(p.in[2] + r * ld + p.d) + p.eps) : 1.f;
#pragma unroll
    for (int i = 0; i < W; ++i) y[i] = q[i] + b[i] + c[i] * scale;
    gn_store<W>(p.out[0] + r * p.d, y, p.d);
  }
}

// ---------------------------------------------------------------- backward

// in {dy [d], C [d+1]} -> out {dC [d+1]}: the mass-normalised read's gradient
template <int W>
__global__ void __launch_bounds__(kGnThreads) gn_out_bwd_kernel(GnRowParams p) {
  const GnRows rs(p);
  const int ld = p.d + 1;
  for (int t = rs.t0 + (threadIdx.x >> 5); t < rs.t1; t += kGnThreads / 32) {
    const size_t r = gn_row(p, rs.bh, t);
    float dy[W], c[W], dc[W];
    gn_load<W>(dy, p.in[0] + r * p.d, p.d);
    gn_load<W>(c, p.in[1] + r * ld, p.d);
    const float scale = 1.f / (__ldg(p.in[1] + r * ld + p.d) + p.eps);
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < W; ++i) {
      dc[i] = dy[i] * scale;
      dot = fmaf(dy[i], c[i], dot);
    }
    dot = gn_warp_sum(dot);
    gn_store<W>(p.out[0] + r * ld, dc, p.d);
    if ((threadIdx.x & 31) == 0) p.out[0][r * ld + p.d] = -dot * scale * scale;
  }
}

// Backward of x -> sigma(x inv(x) - tau) given d(sigma) = dh and an extra
// d(sigma') = dd1 (zero for the read features): returns dx, accumulates the
// threshold gradient.  inv = (mean x^2 + eps)^-1/2.
template <int NL, int W>
__device__ __forceinline__ void gn_rms_act_bwd(float (&dx)[W], const float (&x)[W], const float (&dh)[W],
                                               const float (&dd1)[W], const float (&tau)[W], float (&dtau)[W],
                                               int n, float eps) {
  const float inv = gn_inv_rms<W>(x, n, eps);
  float dn[W], dinv = 0.f;
#pragma unroll
  for (int i = 0; i < W; ++i) {
    float f, d1, d2;
    Act<NL>::eval(fmaf(x[i], inv, -tau[i]), f, d1, d2);
    const bool in = (threadIdx.x & 31) + 32 * i < n;
    dn[i] = in ? fmaf(dh[i], d1, dd1[i] * d2) : 0.f;
    dtau[i] -= dn[i];
    dinv = fmaf(dn[i], x[i], dinv);
  }
  dinv = gn_warp_sum(dinv);
  const float c = dinv * inv * inv * inv / static_cast<float>(n);
#pragma unroll
  for (int i = 0; i < W; ++i) dx[i] = fmaf(inv, dn[i], -c * x[i]);
}

// in {dhq [m], a_q [m], R [m(+1)] or NULL} -> out {da_q [m] (flags bit 1:
// accumulate), dR [m(+1)]}; threshold gradient
template <int NL, int W>
__global__ void __launch_bounds__(kGnThreads) gn_features_bwd_kernel(GnRowParams p) {
  const GnRows rs(p);
  float tau[W], dtau[W];
  gn_tau<W>(tau, p, rs.h);
#pragma unroll
  for (int i = 0; i < W; ++i) dtau[i] = 0.f;
  const bool norm = p.flags & 1, acc = p.flags & 2;
  const int ld = norm ? p.m + 1 : p.m;
  float zero[W];
#pragma unroll
  for (int i = 0; i < W; ++i) zero[i] = 0.f;
  for (int t = rs.t0 + (threadIdx.x >> 5); t < rs.t1; t += kGnThreads / 32) {
    const size_t r = gn_row(p, rs.bh, t);
    float pre[W], rd[W], dh[W], dpre[W], mass;
    const float scale = gn_pre<W>(pre, rd, mass, p, r);
    gn_load<W>(dh, p.in[2] + r * p.m, p.m);
    gn_rms_act_bwd<NL, W>(dpre, pre, dh, zero, tau, dtau, p.m, p.eps);
    gn_store_acc<W>(p.out[0] + r * p.m, dpre, p.m, acc);
    if (p.in[1]) {
      float dr[W], dot = 0.f;
#pragma unroll
      for (int i = 0; i < W; ++i) {
        dr[i] = dpre[i] * scale;
        dot = fmaf(dpre[i], rd[i], dot);
      }
      gn_store<W>(p.out[1] + r * ld, dr, p.m);
      if (norm) {
        dot = gn_warp_sum(dot);
        if ((threadIdx.x & 31) == 0) p.out[1][r * ld + p.m] = -dot * scale * scale;
      }
    }
  }
  if (p.dtau) gn_flush_dtau<W>(p, dtau, rs.h);
}

// in {dh0 [m], a_q [m]} -> out {da_q [m] (flags bit 1: accumulate)}; threshold gradient
template <int W>
__global__ void __launch_bounds__(kGnThreads) gn_query_pre_bwd_kernel(GnRowParams p) {
  const GnRows rs(p);
  float tau[W], dtau[W], zero[W];
  gn_tau<W>(tau, p, rs.h);
#pragma unroll
  for (int i = 0; i < W; ++i) dtau[i] = zero[i] = 0.f;
  const bool acc = p.flags & 2;
  for (int t = rs.t0 + (threadIdx.x >> 5); t < rs.t1; t += kGnThreads / 32) {
    const size_t r = gn_row(p, rs.bh, t);
    float a[W], dh[W], da[W];
    gn_load<W>(dh, p.in[0] + r * p.m, p.m);
    gn_load<W>(a, p.in[1] + r * p.m, p.m);
    gn_rms_act_bwd<TS_GN_RELU2, W>(da, a, dh, zero, tau, dtau, p.m, p.eps);
    gn_store_acc<W>(p.out[0] + r * p.m, da, p.m, acc);
  }
  if (p.dtau) gn_flush_dtau<W>(p, dtau, rs.h);
}

// in {dg [m], a [m]} -> out {du [m]}: du = dg sigma'(p) inv
template <int NL, int W>
__global__ void __launch_bounds__(kGnThreads) gn_write_g_bwd_kernel(GnRowParams p) {
  const GnRows rs(p);
  float tau[W];
  gn_tau<W>(tau, p, rs.h);
  for (int t = rs.t0 + (threadIdx.x >> 5); t < rs.t1; t += kGnThreads / 32) {
    const size_t r = gn_row(p, rs.bh, t);
    float dg[W], a[W], du[W];
    gn_load<W>(dg, p.in[0] + r * p.m, p.m);
    gn_load<W>(a, p.in[1] + r * p.m, p.m);
    const float inv = gn_inv_rms<W>(a, p.m, p.eps);
#pragma unroll
    for (int i = 0; i < W; ++i) {
      float f, d1, d2;
      Act<NL>::eval(fmaf(a[i], inv, -tau[i]), f, d1, d2);
      du[i] = dg[i] * d1 * inv;
    }
    gn_store<W>(p.out[0] + r * p.m, du, p.m);
  }
}

// in {dlam, dlamW, v, k, O, RS [d], hh, kk [1]} -> out {dr [d] (= dv),
// drowsq [d], dk [d] (the k terms outside W1 k), dhh [1]}
template <int W>
__global__ void __launch_bounds__(kGnThreads) gn_write_lam_bwd_kernel(GnRowParams p) {
  const GnRows rs(p);
  for (int t = rs.t0 + (threadIdx.x >> 5); t < rs.t1; t += kGnThreads / 32) {
    const size_t r = gn_row(p, rs.bh, t);
    float dl[W], dw[W], v[W], k[W], o[W], q[W];
    gn_load<W>(dl, p.in[0] + r * p.d, p.d);
    gn_load<W>(dw, p.in[1] + r * p.d, p.d);
    gn_load<W>(v, p.in[2] + r * p.d, p.d);
    gn_load<W>(k, p.in[3] + r * p.d, p.d);
    gn_load<W>(o, p.in[4] + r * p.d, p.d);
    gn_load<W>(q, p.in[5] + r * p.d, p.d);
    const float hh = __ldg(p.in[6] + r), kk = __ldg(p.in[7] + r);
    float dr[W], dden[W], dhh = 0.f, dkk = 0.f;
#pragma unroll
    for (int i = 0; i < W; ++i) {
      const float den = fmaf(kk, q[i], hh) + p.eps;
      const float lam = (v[i] - k[i] - o[i]) / den;
      const float g = dl[i] + dw[i];
      dr[i] = g / den;
      dden[i] = -dr[i] * lam;
      dhh += dden[i];
      dkk = fmaf(dden[i], q[i], dkk);
    }
    dhh = gn_warp_sum(dhh);
    dkk = gn_warp_sum(dkk);
    float drs[W], dk[W];
#pragma unroll
    for (int i = 0; i < W; ++i) {
      drs[i] = dden[i] * kk;
      dk[i] = fmaf(2.f * dkk, k[i], -dr[i]);
    }
    gn_store<W>(p.out[0] + r * p.d, dr, p.d);
    gn_store<W>(p.out[1] + r * p.d, drs, p.d);
    gn_store<W>(p.out[2] + r * p.d, dk, p.d);
    if ((threadIdx.x & 31) == 0) p.out[3][r] = dhh;
  }
}

// in {dh [m], dhO [m] (= W2^T dr), ds2 [m], dhh [1], dg [m], U [m], a [m]}
// -> out {da [m]}; threshold gradient.  The write's h, s = sigma' inv and g =
// sigma' U inv all hang off p = a inv - tau.
template <int NL, int W>
__global__ void __launch_bounds__(kGnThreads) gn_write_pre_bwd_kernel(GnRowParams p) {
  const GnRows rs(p);
  float tau[W], dtau[W];
  gn_tau<W>(tau, p, rs.h);
#pragma unroll
  for (int i = 0; i < W; ++i) dtau[i] = 0.f;
  for (int t = rs.t0 + (threadIdx.x >> 5); t < rs.t1; t += kGnThreads / 32) {
    const size_t r = gn_row(p, rs.bh, t);
    float dh[W], dho[W], ds2[W], dg[W], u[W], a[W];
    gn_load<W>(dh, p.in[0] + r * p.m, p.m);
    gn_load<W>(dho, p.in[1] + r * p.m, p.m);
    gn_load<W>(ds2, p.in[2] + r * p.m, p.m);
    const float dhh = __ldg(p.in[3] + r);
    gn_load<W>(dg, p.in[4] + r * p.m, p.m);
    gn_load<W>(u, p.in[5] + r * p.m, p.m);
    gn_load<W>(a, p.in[6] + r * p.m, p.m);
    const float inv = gn_inv_rms<W>(a, p.m, p.eps);
    // d sigma' and the direct d inv of g = sigma' U inv and s^2 = (sigma' inv)^2
    float dd1[W], dn[W], dinv = 0.f;
#pragma unroll
    for (int i = 0; i < W; ++i) {
      float f, d1, d2;
      Act<NL>::eval(fmaf(a[i], inv, -tau[i]), f, d1, d2);
      const bool in = (threadIdx.x & 31) + 32 * i < p.m;
      const float s = d1 * inv;
      const float ds = 2.f * s * ds2[i];
      dd1[i] = fmaf(dg[i] * u[i], inv, ds * inv);
      dinv = fmaf(dg[i] * d1, u[i], fmaf(ds, d1, dinv));
      const float dht = fmaf(2.f * dhh, f, dh[i] - dho[i]);
      dn[i] = in ? fmaf(dht, d1, dd1[i] * d2) : 0.f;
      dtau[i] -= dn[i];
      dinv = fmaf(dn[i], a[i], dinv);
    }
    dinv = gn_warp_sum(dinv);
    const float c = dinv * inv * inv * inv / static_cast<float>(p.m);
    float da[W];
#pragma unroll
    for (int i = 0; i < W; ++i) da[i] = fmaf(inv, dn[i], -c * a[i]);
    gn_store<W>(p.out[0] + r * p.m, da, p.m);
  }
  if (p.dtau) gn_flush_dtau<W>(p, dtau, rs.h);
}

// ---------------------------------------------------------------- q/k/v preparation

// The GN mixer's streams from its fused projection (block.py:577-599 of the
// reference): q and k rotated on their first `rot` channels (adjacent pairs,
// phases cos/sin [T][rot/2]) and L2-normalised, x / max(|x|, eps); v copied.
// src is the projection [B,T,3,H,d]; q, k, v are [B,H,T,d].
struct GnPrepParams {
  int B, H, T, d, rot;
  float eps;
  const float* src;
  const float* cos;
  const float* sin;
  float* q;
  float* k;
  float* v;
  const float* dq;
  const float* dk;
  const float* dv;
  float* dsrc;
};

// the rotation (sign +1) or its transpose (sign -1) of the lane's slots
template <int W>
__device__ __forceinline__ void gn_rotate(float (&x)[W], const GnPrepParams& p, int t, float sign) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int i = 0; i < W; ++i) {
    const int c = lane + 32 * i;
    const float other = __shfl_xor_sync(0xffffffffu, x[i], 1);
    if (c < p.rot) {
      const int j = c >> 1;
      const float cs = __ldg(p.cos + static_cast<size_t>(t) * (p.rot >> 1) + j);
      const float sn = sign * __ldg(p.sin + static_cast<size_t>(t) * (p.rot >> 1) + j);
      x[i] = (c & 1) ? fmaf(other, sn, x[i] * cs) : fmaf(-other, sn, x[i] * cs);
    }
  }
}

template <int W>
__global__ void __launch_bounds__(kGnThreads) gn_prep_fwd_kernel(GnPrepParams p) {
  const int bh = blockIdx.y, b = bh / p.H, h = bh % p.H;
  const int t0 = blockIdx.x * kGnRowsPerCta, t1 = min(p.T, t0 + kGnRowsPerCta);
  for (int t = t0 + (threadIdx.x >> 5); t < t1; t += kGnThreads / 32) {
    const float* row = p.src + ((static_cast<size_t>(b) * p.T + t) * 3 * p.H + h) * p.d;
    const size_t o = (static_cast<size_t>(bh) * p.T + t) * p.d;
    for (int which = 0; which < 2; ++which) {
      float x[W];
      gn_load<W>(x, row + static_cast<size_t>(which) * p.H * p.d, p.d);
      gn_rotate<W>(x, p, t, 1.f);
      float n = 0.f;
#pragma unroll
      for (int i = 0; i < W; ++i) n = fmaf(x[i], x[i], n);
      const float inv = 1.f / fmaxf(sqrtf(gn_warp_sum(n)), p.eps);
#pragma unroll
      for (int i = 0; i < W; ++i) x[i] *= inv;
      gn_store<W>((which ? p.k : p.q) + o, x, p.d);
    }
    float x[W];
    gn_load<W>(x, row + static_cast<size_t>(2) * p.H * p.d, p.d);
    gn_store<W>(p.v + o, x, p.d);
  }
}

template <int W>
__global__ void __launch_bounds__(kGnThreads) gn_prep_bwd_kernel(GnPrepParams p) {
  const int bh = blockIdx.y, b = bh / p.H, h = bh % p.H;
  const int t0 = blockIdx.x * kGnRowsPerCta, t1 = min(p.T, t0 + kGnRowsPerCta);
  for (int t = t0 + (threadIdx.x >> 5); t < t1; t += kGnThreads / 32) {
    const size_t srow = ((static_cast<size_t>(b) * p.T + t) * 3 * p.H + h) * p.d;
    const size_t o = (static_cast<size_t>(bh) * p.T + t) * p.d;
    for (int which = 0; which < 2; ++which) {
      float x[W], g[W];
      gn_load<W>(x, p.src + srow + static_cast<size_t>(which) * p.H * p.d, p.d);
      gn_load<W>(g, (which ? p.dk : p.dq) + o, p.d);
      gn_rotate<W>(x, p, t, 1.f);
      float n = 0.f, dot = 0.f;
#pragma unroll
      for (int i = 0; i < W; ++i) {
        n = fmaf(x[i], x[i], n);
        dot = fmaf(x[i], g[i], dot);
      }
      n = sqrtf(gn_warp_sum(n));
      dot = gn_warp_sum(dot);
      // out = x / max(|x|, eps): below the floor the divisor is a constant
      const float inv = 1.f / fmaxf(n, p.eps);
      const float c = n > p.eps ? dot * inv * inv * inv : 0.f;
#pragma unroll
      for (int i = 0; i < W; ++i) g[i] = fmaf(g[i], inv, -c * x[i]);
      gn_rotate<W>(g, p, t, -1.f);
      gn_store<W>(p.dsrc + srow + static_cast<size_t>(which) * p.H * p.d, g, p.d);
    }
    float g[W];
    gn_load<W>(g, p.dv + o, p.d);
    gn_store<W>(p.dsrc + srow + static_cast<size_t>(2) * p.H * p.d, g, p.d);
  }
}

int launch_gn_prep(const GnPrepParams& p, bool backward, cudaStream_t s) {
  if (p.B <= 0 || p.H <= 0 || p.T <= 0) return TS_OK;
  const dim3 grid(ceil_div(p.T, kGnRowsPerCta), p.B * p.H);
  if (p.d <= 128) {
    if (backward) gn_prep_bwd_kernel<4><<<grid, kGnThreads, 0, s>>>(p);
    else gn_prep_fwd_kernel<4><<<grid, kGnThreads, 0, s>>>(p);
  } else {
    if (backward) gn_prep_bwd_kernel<8><<<grid, kGnThreads, 0, s>>>(p);
    else gn_prep_fwd_kernel<8><<<grid, kGnThreads, 0, s>>>(p);
  }
  return check_launch(backward ? "gn_prep_bwd_kernel" : "gn_prep_fwd_kernel");
}

// ---------------------------------------------------------------- launch

template <int W>
int launch_gn_rows_w(const GnRowParams& p, int stage, cudaStream_t s) {
  const dim3 grid(ceil_div(p.T, kGnRowsPerCta), p.B * p.H);
#define TS_GN_NL(KERNEL)                                                                     \
  switch (p.nonlin) {                                                                        \
    case TS_GN_RELU2: KERNEL<TS_GN_RELU2, W><<<grid, kGnThreads, 0, s>>>(p); break;          \
    case TS_GN_SILU: KERNEL<TS_GN_SILU, W><<<grid, kGnThreads, 0, s>>>(p); break;            \
    default: KERNEL<TS_GN_TANH, W><<<grid, kGnThreads, 0, s>>>(p); break;                    \
  }                                                                                          \
  return check_launch(#KERNEL);
  switch (stage) {
    case TS_GN_WRITE_PRE: TS_GN_NL(gn_write_pre_kernel)
    case TS_GN_WRITE_G: TS_GN_NL(gn_write_g_kernel)
    case TS_GN_FEATURES: TS_GN_NL(gn_features_kernel)
    case TS_GN_FEATURES_BWD: TS_GN_NL(gn_features_bwd_kernel)
    case TS_GN_WRITE_G_BWD: TS_GN_NL(gn_write_g_bwd_kernel)
    case TS_GN_WRITE_PRE_BWD: TS_GN_NL(gn_write_pre_bwd_kernel)
    case TS_GN_WRITE_LAM:
      gn_write_lam_kernel<W><<<grid, kGnThreads, 0, s>>>(p);
      return check_launch("gn_write_lam_kernel");
    case TS_GN_QUERY_PRE:
      gn_query_pre_kernel<W><<<grid, kGnThreads, 0, s>>>(p);
      return check_launch("gn_query_pre_kernel");
    case TS_GN_OUT:
      gn_out_kernel<W><<<grid, kGnThreads, 0, s>>>(p);
      return check_launch("gn_out_kernel");
    case TS_GN_OUT_BWD:
      gn_out_bwd_kernel<W><<<grid, kGnThreads, 0, s>>>(p);
      return check_launch("gn_out_bwd_kernel");
    case TS_GN_QUERY_PRE_BWD:
      gn_query_pre_bwd_kernel<W><<<grid, kGnThreads, 0, s>>>(p);
      return check_launch("gn_query_pre_bwd_kernel");
    case TS_GN_WRITE_LAM_BWD:
      gn_write_lam_bwd_kernel<W><<<grid, kGnThreads, 0, s>>>(p);
      return check_launch("gn_write_lam_bwd_kernel");
    default:
      return set_error(TS_ERR_VALUE, "gn_rows: unknown stage %d", stage);
  }
#undef TS_GN_NL
}

int launch_gn_rows(const GnRowParams& p, int stage, cudaStream_t s) {
  if (p.B <= 0 || p.H <= 0 || p.T <= 0) return TS_OK;
  return max(p.d, p.m) <= 128 ? launch_gn_rows_w<4>(p, stage, s) : launch_gn_rows_w<8>(p, stage, s);
}

}  // namespace ts
