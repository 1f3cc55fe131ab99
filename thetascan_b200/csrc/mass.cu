// Per-feature mass of the feature-mass read (reference engine.py:443-456):
// each view divides the query features by its own cumulative key-feature mass
//   mass_t[f] = sum_{j<=t} w(t-j) phi_k[j][f]
// (view.mass_cum, interface.py:216-230, 278-279, 306-307; ema_cumsum,
// interface.py:58-93) before an unnormalized scan reads it.  The weights are
// those of the view: 1 (plain sum), alpha^(t-j) (recency) or 1 - alpha^(t-j)
// (stale, = prefix sum - recency mass), formed by recursions whose terms are
// all nonnegative:
//   D_t = alpha D_{t-1} + x_t                      (recency mass)
//   X_t = X_{t-1} + (1 - alpha) D_{t-1}            (stale mass, no cancellation)
// Forward output: q_scaled_t = phi_q_t / (mass_t + eps), bf16 (or f32 for a
// float32 scan).
//
// Backward, with g = d q_scaled:
//   d phi_q_t  += g_t / (mass_t + eps)
//   d mass_t    = -g_t q_scaled_t / (mass_t + eps)      (q_scaled as the scan read it)
//   d phi_k_j  += sum_{t>=j} w(t-j) d mass_t        (reverse recursions)
//   d la       += sum_t d mass_t dmass_t/dla,  dD_t/dla = F_t = alpha (F_{t-1} + D_{t-1}),
//                 dX_t/dla = -F_t
// The sweep over tokens is sequential per feature; a thread owns two adjacent
// features (one bf16x2 word, so a warp touches 128 contiguous bytes per row)
// and loads kMassBatch rows ahead of the recursion.  This path is HBM/latency
// bound elementwise work: no tensor cores.
#include "capi_internal.h"
#include "common.cuh"

namespace ts {

struct MassParams {
  int B, H, T, m;
  const __nv_bfloat16* phi_k;  // [B,H,T,m]
  const __nv_bfloat16* phi_q;  // [B,H,T,m]
  const float* phi_q32;        // [B,H,T,m] f32, read instead of phi_q when set
  const float* la;             // [H] or null (plain prefix sum)
  int stale;
  float eps;
  void* qs;                    // [B,H,T,m] out, bf16 or (qs_f32) f32
  int qs_f32;
  // backward
  const void* dqs;
  int dqs_bf16;
  float* dphi_q;               // accumulated
  float* dphi_k;               // accumulated
  float* dla;                  // accumulated, or null
  float* dmass;                // scratch [B,H,T,m]
};

namespace {

constexpr int kMassBatch = 8;

__device__ __forceinline__ float2 ld_bf2(const __nv_bfloat16* p) {
  const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(p);
  return __bfloat1622float2(v);
}

__device__ __forceinline__ float2 ld_query(const MassParams& p, size_t o) {
  return p.phi_q32 ? *reinterpret_cast<const float2*>(p.phi_q32 + o) : ld_bf2(p.phi_q + o);
}

// One token of the mass recursion for one feature; returns mass_t.
struct MassState {
  float D = 0.f, X = 0.f, F = 0.f;
  __device__ __forceinline__ float step(float x, float alpha, float open, bool decayed, bool stale, bool with_f) {
    if (!decayed) {
      D += x;
      return D;
    }
    if (with_f) F = alpha * (F + D);
    if (stale) X += open * D;
    D = alpha * D + x;
    return stale ? X : D;
  }
};

}  // namespace

__global__ void __launch_bounds__(256) mass_fwd_kernel(MassParams p) {
  const int f2 = threadIdx.x;            // feature pair
  const int bh = blockIdx.x;
  if (2 * f2 >= p.m) return;
  const int h = bh % p.H;
  const bool decayed = p.la != nullptr;
  const float la = decayed ? __ldg(p.la + h) : 0.f;
  const float alpha = __expf(la), open = -expm1f(la);
  const size_t base = static_cast<size_t>(bh) * p.T * p.m + 2 * f2;
  MassState s0, s1;
  for (int t0 = 0; t0 < p.T; t0 += kMassBatch) {
    float2 xk[kMassBatch], xq[kMassBatch];
#pragma unroll
    for (int i = 0; i < kMassBatch; ++i) {
      if (t0 + i < p.T) {
        xk[i] = ld_bf2(p.phi_k + base + static_cast<size_t>(t0 + i) * p.m);
        xq[i] = ld_query(p, base + static_cast<size_t>(t0 + i) * p.m);
      }
    }
#pragma unroll
    for (int i = 0; i < kMassBatch; ++i) {
      if (t0 + i >= p.T) break;
      const float m0 = s0.step(xk[i].x, alpha, open, decayed, p.stale, false);
      const float m1 = s1.step(xk[i].y, alpha, open, decayed, p.stale, false);
      const size_t o = base + static_cast<size_t>(t0 + i) * p.m;
      const float2 qv = make_float2(xq[i].x / (m0 + p.eps), xq[i].y / (m1 + p.eps));
      if (p.qs_f32)
        *reinterpret_cast<float2*>(static_cast<float*>(p.qs) + o) = qv;
      else
        *reinterpret_cast<__nv_bfloat162*>(static_cast<__nv_bfloat16*>(p.qs) + o) = __float22bfloat162_rn(qv);
    }
  }
}

__global__ void __launch_bounds__(256) mass_bwd_kernel(MassParams p) {
  __shared__ float red[8];
  const int f2 = threadIdx.x;
  const int bh = blockIdx.x;
  const bool active = 2 * f2 < p.m;
  const int h = bh % p.H;
  const bool decayed = p.la != nullptr;
  const bool want = decayed && p.dla != nullptr;
  const float la = decayed ? __ldg(p.la + h) : 0.f;
  const float alpha = __expf(la), open = -expm1f(la);
  const size_t base = static_cast<size_t>(bh) * p.T * p.m + 2 * f2;
  float acc = 0.f;
  if (active) {
    // sweep 1, forward: the mass again, d phi_q, d mass and the la terms
    MassState s0, s1;
    for (int t0 = 0; t0 < p.T; t0 += kMassBatch) {
      float2 xk[kMassBatch], xq[kMassBatch], g[kMassBatch];
#pragma unroll
      for (int i = 0; i < kMassBatch; ++i) {
        if (t0 + i < p.T) {
          const size_t o = base + static_cast<size_t>(t0 + i) * p.m;
          xk[i] = ld_bf2(p.phi_k + o);
          xq[i] = ld_query(p, o);
          g[i] = p.dqs_bf16 ? ld_bf2(static_cast<const __nv_bfloat16*>(p.dqs) + o)
                            : *reinterpret_cast<const float2*>(static_cast<const float*>(p.dqs) + o);
        }
      }
#pragma unroll
      for (int i = 0; i < kMassBatch; ++i) {
        if (t0 + i >= p.T) break;
        const size_t o = base + static_cast<size_t>(t0 + i) * p.m;
        const float m0 = s0.step(xk[i].x, alpha, open, decayed, p.stale, want);
        const float m1 = s1.step(xk[i].y, alpha, open, decayed, p.stale, want);
        const float i0 = 1.f / (m0 + p.eps), i1 = 1.f / (m1 + p.eps);
        float2* dq = reinterpret_cast<float2*>(p.dphi_q + o);
        float2 cur = *dq;
        cur.x += g[i].x * i0;
        cur.y += g[i].y * i1;
        *dq = cur;
        // d mass from the quotient the scan read (the forward's value, bf16-
        // rounded for a bf16 scan): its gradient then cancels against the
        // scan's d phi_k as the quotient rule does, instead of leaving a 2^-9
        // residual of each term
        float2 qs = make_float2(xq[i].x / (m0 + p.eps), xq[i].y / (m1 + p.eps));
        if (!p.qs_f32) qs = __bfloat1622float2(__float22bfloat162_rn(qs));
        const float dm0 = -g[i].x * qs.x * i0, dm1 = -g[i].y * qs.y * i1;
        *reinterpret_cast<float2*>(p.dmass + o) = make_float2(dm0, dm1);
        if (want) {
          // F after this token's step is dD_t/dla; the stale mass has -F
          const float sgn = p.stale ? -1.f : 1.f;
          acc += sgn * (dm0 * s0.F + dm1 * s1.F);
        }
      }
    }
    // sweep 2, reverse: d phi_k_j = sum_{t>=j} w(t-j) d mass_t
    float E0 = 0.f, E1 = 0.f, Y0 = 0.f, Y1 = 0.f;
    for (int t1 = p.T - 1; t1 >= 0; t1 -= kMassBatch) {
      float2 dm[kMassBatch];
#pragma unroll
      for (int i = 0; i < kMassBatch; ++i)
        if (t1 - i >= 0) dm[i] = *reinterpret_cast<const float2*>(p.dmass + base + static_cast<size_t>(t1 - i) * p.m);
#pragma unroll
      for (int i = 0; i < kMassBatch; ++i) {
        const int t = t1 - i;
        if (t < 0) break;
        float d0, d1;
        if (!decayed) {
          E0 += dm[i].x;
          E1 += dm[i].y;
          d0 = E0;
          d1 = E1;
        } else if (p.stale) {
          // Y_j = Y_{j+1} + (1 - alpha) E_{j+1},  E_j = alpha E_{j+1} + d mass_j
          Y0 += open * E0;
          Y1 += open * E1;
          E0 = alpha * E0 + dm[i].x;
          E1 = alpha * E1 + dm[i].y;
          d0 = Y0;
          d1 = Y1;
        } else {
          E0 = alpha * E0 + dm[i].x;
          E1 = alpha * E1 + dm[i].y;
          d0 = E0;
          d1 = E1;
        }
        float2* dk = reinterpret_cast<float2*>(p.dphi_k + base + static_cast<size_t>(t) * p.m);
        float2 cur = *dk;
        cur.x += d0;
        cur.y += d1;
        *dk = cur;
      }
    }
  }
  if (want) {
    float v = acc;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    if (threadIdx.x == 0) {
      float sum = 0.f;
      for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) sum += red[w];
      atomicAdd(p.dla + h, sum);
    }
  }
}

static int mass_threads(const MassParams& p) { return ((p.m / 2 + 31) / 32) * 32; }

int launch_mass_fwd(const MassParams& p, cudaStream_t s) {
  mass_fwd_kernel<<<p.B * p.H, mass_threads(p), 0, s>>>(p);
  return check_launch("mass_fwd_kernel");
}

int launch_mass_bwd(const MassParams& p, cudaStream_t s) {
  mass_bwd_kernel<<<p.B * p.H, mass_threads(p), 0, s>>>(p);
  return check_launch("mass_bwd_kernel");
}

}  // namespace ts
