// Per-token feature maps of the kernel-family write and read, fused around a
// tcgen05 projection.  Forward, per 128-token tile of x in {k, q}:
//   a   = x W1^T                       (tcgen05, TMEM, f32)
//   pre = a * rsqrt(mean(a^2) + eps)   (RMSNorm, reference norms.py:5-8)
//   phi = map(pre)                     (kernel_features.py:116-135 relu2 ridge,
//                                       :73-113 softmax partition, with
//                                       :43-70 relative sparsity,
//                                       :138-230 projected cubic B-spline)
// and for q additionally y0 = q + W2 phi (the slow decode of engine.py:524 plus
// the residual of engine.py:526).  The backward recomputes a and phi and
// produces dx = dA W1 (+ dy for q), dW1 += dA^T x, dW2 += dy^T phi and the
// gradients of the per-head / per-feature controls.
//
// Two threads own one token row (threads t and t+128 read the same TMEM lane
// quadrant and split the row's columns into alternating 16-column chunks);
// row reductions combine the two halves through shared memory.
#include "capi_internal.h"
#include "common.cuh"

namespace ts {

// kSoftmaxSparse: the softmax partition with a relative sparsity mode
// (FeatParams.sparse_mode); the host passes kind softmax.
enum FeatureKind { kRelu2 = 0, kSoftmax = 1, kBspline = 2, kSoftmaxSparse = 3 };
constexpr int kMaxBasis = 16;

struct FeatParams {
  int B, H, T;
  int d, dP;          // head width, padded to 16
  int P, PP, PM;      // projections, padded to 16 and to 128
  int m, mP, mM;      // feature width, padded to 16 and to 128
  int kind;
  float eps;
  int nsel, sel0;     // selections processed (0 = k, 1 = q)
  const __nv_bfloat16* x[2];
  long long xs[2][3];
  const __nv_bfloat16* W1;  // [H, P, d]
  const __nv_bfloat16* W2;  // [H, d, m] (may be null)
  const float* bias;        // [H, m] or null
  const float* thr;         // [H] or null
  const float* gain;        // [H] or [H, m] or null
  int gain_mode;            // 0 scalar, 1 per head, 2 per feature
  float gain_scalar;
  const float* scale;       // [H] or null
  float scale_scalar;
  int nb;
  float bound;
  // forward outputs
  __nv_bfloat16* phi[2];    // [B, H, T, m]
  float* phi_q32;           // [B, H, T, m] f32 copy of phi_q, or null
  int dW2_t;                // backward: dW2 accumulated as [H, m, d] (vector atomics)
  float* y0;                // [B, H, T, d] or null (q only)
  // backward
  const void* dphi[2];      // [B, H, T, m], f32 or bf16
  int dphi_bf16;
  const float* dy;          // [B, H, T, d] (q only) or null
  const __nv_bfloat16* dyb; // or bf16 strided view of it
  long long dys[3];
  float* dx[2];             // [B, H, T, d]
  float* dW1;               // [H, P, d]
  float* dW2;               // [H, d, m]
  float* dbias;             // [H, m]
  float* dthr;              // [H]
  float* dgain;             // [H] or [H, m]
  float* dscale;            // [H]
  // fused row prologue (raw projections in x): rotation tables [pos0 + T, rot/2]
  int rot, pos0, l2norm;
  float neps;
  const float* rcos;
  const float* rsin;
  // bf16 strided row-gradient outputs in place of the f32 dx
  __nv_bfloat16* dxb[2];
  long long dxs[2][3];
  // relative sparsity of the softmax partition (kernel_features.py:43-70,
  // 95-113): mode 1 relative_soft, 2 relative_st, 3 relative_st_blend
  int sparse_mode;
  float temperature;
  const float* rho;         // [H] relative cutoff in (0, 1)
  const float* alpha;       // [H] dense-to-sparse blend (mode 3)
  float* drho;              // [H], accumulated
  float* dalpha;            // [H], accumulated
};

// Kernels are instantiated per feature kind KF & kKindMask; with kPlainBit
// set the map has no score bias, no relu2 threshold, one fixed softmax gain
// and no column tail (P == PP), so the per-element controls and bounds
// checks compile away.
constexpr int kKindMask = 7;
constexpr int kPlainBit = 8;

template <bool kPlain = false>
__device__ __forceinline__ float ctl_bias(const FeatParams& p, int h, int i) {
  if constexpr (kPlain) return 0.f;
  return p.bias ? __ldg(p.bias + h * p.m + i) : 0.f;
}
template <bool kPlain = false>
__device__ __forceinline__ float ctl_gain(const FeatParams& p, int h, int i) {
  if constexpr (kPlain) return p.gain_scalar;
  return p.gain_mode == 0 ? p.gain_scalar : p.gain_mode == 1 ? __ldg(p.gain + h) : __ldg(p.gain + h * p.m + i);
}
template <bool kPlain = false>
__device__ __forceinline__ float ctl_thr(const FeatParams& p, int h) {
  if constexpr (kPlain) return 0.f;
  return p.thr ? __ldg(p.thr + h) : 0.f;
}

// Packed f32x2 arithmetic (two lanes per instruction; each lane rounds as
// the scalar operation does) for the plain relu2 loops.
__device__ __forceinline__ float2 f2(float x, float y) { return make_float2(x, y); }
__device__ __forceinline__ float2 relu2_u(float2 a, float2 inv) {
  const float2 t = __fmul2_rn(a, inv);
  return f2(fmaxf(t.x, 0.f), fmaxf(t.y, 0.f));
}
__device__ __forceinline__ float ctl_scale(const FeatParams& p, int h) {
  return p.scale ? __ldg(p.scale + h) : p.scale_scalar;
}

// Cubic (degree-3) open-uniform B-spline basis at x with its derivative, by
// the Cox--de Boor recursion on knots [-b]*4, uniform interior, [b]*4
// (reference kernel_features.py:138-205: half-open spans, zero-width spans
// dropped, clamp to [-b, nextafter(b, -b)], negatives clamped, renormalised).
// At a coordinate in knot span j (knot[j] <= x < knot[j+1]) only the degree-3
// functions j-3 .. j can be nonzero, so the recursion runs on that window of
// four; every term it skips is an exact zero, which leaves the values, the
// derivatives and the normalising sums what the recursion over all functions
// gives.  Writes val/der of functions first .. first+3 (first = j - 3);
// `inside` is false when the coordinate was clamped (zero derivative).
__device__ __forceinline__ float bspline_knot(int i, int nb, float bound, float step) {
  return i <= 3 ? -bound : (i >= nb ? bound : -bound + static_cast<float>(i - 3) * step);
}

// The knots (nb + 4 of them, nb <= 16) and the reciprocals of the knot
// differences the recursion divides by, rd[o-1][i] = 1 / (knot[i+o] - knot[i])
// (0 where the difference is zero: the reference drops those terms), built
// once per CTA so that the recursion multiplies instead of dividing.
constexpr int kMaxKnots = 20;
struct SplineTable {
  float knot[kMaxKnots];
  float rd[3][kMaxKnots];
  float inv_step;
};

__device__ void build_spline_table(SplineTable& t, int nb, float bound) {
  const float step = 2.f * bound / static_cast<float>(nb - 3);
  const int nk = nb + 4;
  for (int i = threadIdx.x; i < nk; i += blockDim.x) t.knot[i] = bspline_knot(i, nb, bound, step);
  __syncthreads();
  for (int e = threadIdx.x; e < 3 * nk; e += blockDim.x) {
    const int o = 1 + e / nk, i = e % nk;
    float r = 0.f;
    if (i + o < nk) {
      const float dl = t.knot[i + o] - t.knot[i];
      r = dl > 0.f ? 1.f / dl : 0.f;
    }
    t.rd[o - 1][i] = r;
  }
  if (threadIdx.x == 0) t.inv_step = 1.f / step;
  __syncthreads();
}

__device__ __forceinline__ void bspline_local(float c, int nb, float bound, const SplineTable& t, float* val,
                                              float* der, int& first, bool& inside) {
  const float hi = nextafterf(bound, -bound);
  inside = (c >= -bound) && (c <= bound);
  float x = fminf(fmaxf(c, -bound), bound);
  if (x > hi) x = hi;
  int j = 3 + static_cast<int>(floorf((x + bound) * t.inv_step));
  j = min(max(j, 3), nb - 1);
  while (j > 3 && x < t.knot[j]) --j;
  while (j < nb - 1 && x >= t.knot[j + 1]) ++j;
  float B[4] = {0.f, 0.f, 0.f, 1.f}, D[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int o = 1; o <= 3; ++o) {
#pragma unroll
    for (int s = 3 - o; s < 4; ++s) {
      const int i = j - 3 + s;
      const float rl = t.rd[o - 1][i], rr = t.rd[o - 1][i + 1];
      const float L = (x - t.knot[i]) * rl;
      const float R = (t.knot[i + o + 1] - x) * rr;
      const float b1 = s < 3 ? B[s + 1] : 0.f, d1 = s < 3 ? D[s + 1] : 0.f;
      const float nb_ = L * B[s] + R * b1;
      const float nd_ = rl * B[s] + L * D[s] - rr * b1 + R * d1;
      B[s] = nb_;
      D[s] = nd_;
    }
  }
  float S = 0.f, dS = 0.f;
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    if (B[s] < 0.f) {
      B[s] = 0.f;
      D[s] = 0.f;
    }
    S += B[s];
    dS += D[s];
  }
  const float invS = 1.f / fmaxf(S, 1.17549435e-38f);
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    val[s] = B[s] * invS;
    der[s] = (D[s] - B[s] * dS * invS) * invS;
  }
  first = j - 3;
}

// Element idx (0..3) of a 4-vector by value selects (no local memory).
__device__ __forceinline__ float pick4(const float* v, int idx) {
  return idx == 0 ? v[0] : idx == 1 ? v[1] : idx == 2 ? v[2] : v[3];
}

// B-spline projections are dealt out to the kParts threads of a row: thread
// part takes projections part, part + kParts, ... (P <= 32, two 16-column
// chunks of the projection accumulator at most).
constexpr int kMaxSplineOwn = 32 / kParts;

// ------------------------------------------------------------------ shared tile setup

struct FeatTiles {
  Tile x, w1, phi, w2, dy, da;
};

__device__ __forceinline__ void load_weight_rows(const Tile& t, const __nv_bfloat16* __restrict__ src, int rows,
                                                 int cols) {
  load_tile(t, src, cols, rows, cols);
}

// a = x W1^T for this tile into TMEM columns [t_a, t_a + PP).
__device__ __forceinline__ void project(const FeatParams& p, MmaCtx& ctx, const FeatTiles& tl, uint32_t t_a) {
  ctx.run([&] { gemm_issue(t_a, kmajor(tl.x), kmajor(tl.w1), p.PP, p.dP, false); });
}

// Row statistics of the feature map for this thread's row.
struct RowState {
  float inv;    // 1 / rms(a)
  float mass;   // relu2: sum of squared ReLU; softmax: sum of exp
  float mx;     // softmax: max logit
  float dphi;   // with a gradient: sum_j g_j phi_j (relu2 / softmax)
  // With a gradient, row totals of the RMSNorm backward and the per-head
  // controls: dot_a = sum_j dpre_j a_j, dthr = -sum_j dpre_j (relu2),
  // dgain = sum_j dpre_j sc_j / gain_j (softmax, one gain per head).
  float dot_a, dthr, dgain;
  // relative sparsity: sparse normaliser Z, per-column share of the max's
  // gradient, sum g dense, sum g sparse, sum of the margin gradients,
  // log of the clamped cutoff and the blend
  float z, dmx, Sd, Ss, dmarg, lrho, alpha;
};

struct NoGrad {
  __device__ __forceinline__ void operator()(int, float*) const {}
};

// ---- relative sparsity (kernel_features.py:43-70): logits l_j = gain_j
// (pre_j + b_j), shifted s_j = l_j - max l, margin m_j = s_j - log rho_h,
// gate = sigmoid(m / temperature) (soft) or [m >= 0] with the sigmoid's
// derivative (straight-through), sparse_j = e^{s_j} gate_j / max(sum_k
// e^{s_k} gate_k, eps), phi = sparse, or dense + alpha (sparse - dense).
__device__ __forceinline__ float softmax_logit(const FeatParams& p, int h, int i, float a, float inv) {
  return ctl_gain<false>(p, h, i) * (a * inv + ctl_bias<false>(p, h, i));
}

// sigmoid(z) and its derivative from w = e^{-|z|}: s(1 - s) = w / (1 + w)^2
// keeps its relative precision where s is within a few ulp of 1 (the top
// features, whose margin is about -log rho; 1 - s formed by subtraction loses
// most of its digits there).
__device__ __forceinline__ void sparse_gate(const FeatParams& p, float margin, float& gate, float& dgate) {
  const float z = margin / p.temperature;
  const float w = expf(-fabsf(z));
  const float r = 1.f / (1.f + w);
  const float sg = z >= 0.f ? r : w * r;
  gate = p.sparse_mode == 1 ? sg : (margin >= 0.f ? 1.f : 0.f);
  dgate = w * r * r / p.temperature;
}

// d loss / d l_j of one column without the share of the max's gradient
// (dl), and its parts through the shifted logit (dshift) and the margin.
struct SparseTerms {
  float dl, dshift, dmargin;
};
__device__ __forceinline__ SparseTerms sparse_terms(const FeatParams& p, const RowState& s, float g, float l) {
  const float ex = expf(l - s.mx);
  float gt, dgt;
  sparse_gate(p, l - s.mx - s.lrho, gt, dgt);
  const bool blend = p.sparse_mode == 3;
  const float cd = blend ? 1.f - s.alpha : 0.f, cs = blend ? s.alpha : 1.f;
  const float dw = (cs * g - (s.z >= p.eps ? cs * s.Ss : 0.f)) / fmaxf(s.z, p.eps);
  SparseTerms t;
  t.dmargin = dw * ex * dgt;
  t.dshift = dw * ex * gt + t.dmargin;
  t.dl = cd * (ex / s.mass) * (g - s.Sd) + t.dshift;
  return t;
}

// Row statistics of the sparse map: ss, then the max (and how many columns
// hold it), then E = sum e and Z = sum e gate; with a gradient also sum g
// dense, sum g sparse, and the row totals of dpre_j = gain_j dl_j that the
// RMSNorm and control backward need, with the max's gradient -sum dshift
// shared by the columns that hold the max (as torch's amax backward).
template <int KF, bool kWithGrad, class Grad>
__device__ RowState row_stats_sparse(const FeatParams& p, uint32_t ta_row, int h, float* pair, Grad grad16) {
  const int part = my_part();
  RowState s{0.f, 0.f, -INFINITY, 0.f, 0.f, 0.f, 0.f};
  float ss = 0.f;
  for (int c = 16 * part; c < p.PP; c += kChunkStep) {
    float a[16];
    tmem_ld16(ta_row + c, a);
#pragma unroll
    for (int e = 0; e < 16; ++e) ss += a[e] * a[e];
  }
  ss = row_pair_sum(ss, pair);
  s.inv = rsqrtf(ss / static_cast<float>(p.P) + p.eps);
  s.lrho = logf(fminf(fmaxf(__ldg(p.rho + h), p.eps), 1.f - p.eps));
  s.alpha = p.sparse_mode == 3 ? __ldg(p.alpha + h) : 1.f;
  float m = -INFINITY;
  for (int c = 16 * part; c < p.PP; c += kChunkStep) {
    float a[16];
    tmem_ld16(ta_row + c, a);
#pragma unroll
    for (int e = 0; e < 16; ++e)
      if (c + e < p.P) m = fmaxf(m, softmax_logit(p, h, c + e, a[e], s.inv));
  }
  s.mx = row_pair_max(m, pair);
  float E = 0.f, Z = 0.f, cnt = 0.f;
  for (int c = 16 * part; c < p.PP; c += kChunkStep) {
    float a[16];
    tmem_ld16(ta_row + c, a);
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      if (c + e >= p.P) continue;
      const float l = softmax_logit(p, h, c + e, a[e], s.inv);
      const float ex = expf(l - s.mx);
      float gt, dgt;
      sparse_gate(p, l - s.mx - s.lrho, gt, dgt);
      E += ex;
      Z += ex * gt;
      cnt += l == s.mx ? 1.f : 0.f;
    }
  }
  s.mass = row_pair_sum(E, pair);
  s.z = row_pair_sum(Z, pair);
  cnt = row_pair_sum(cnt, pair);
  if constexpr (kWithGrad) {
    const float invE = 1.f / s.mass, invZ = 1.f / fmaxf(s.z, p.eps);
    float Sd = 0.f, Ss = 0.f;
    for (int c = 16 * part; c < p.PP; c += kChunkStep) {
      float a[16], g[16];
      tmem_ld16(ta_row + c, a);
      grad16(c, g);
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        if (c + e >= p.P) continue;
        const float l = softmax_logit(p, h, c + e, a[e], s.inv);
        const float ex = expf(l - s.mx);
        float gt, dgt;
        sparse_gate(p, l - s.mx - s.lrho, gt, dgt);
        Sd += g[e] * ex * invE;
        Ss += g[e] * ex * gt * invZ;
      }
    }
    s.Sd = row_pair_sum(Sd, pair);
    s.Ss = row_pair_sum(Ss, pair);
    float dsh = 0.f, dmarg = 0.f, dot = 0.f, dgn = 0.f;
    for (int c = 16 * part; c < p.PP; c += kChunkStep) {
      float a[16], g[16];
      tmem_ld16(ta_row + c, a);
      grad16(c, g);
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const int i = c + e;
        if (i >= p.P) continue;
        const float l = softmax_logit(p, h, i, a[e], s.inv);
        const SparseTerms t = sparse_terms(p, s, g[e], l);
        dsh += t.dshift;
        dmarg += t.dmargin;
        dot += ctl_gain<false>(p, h, i) * t.dl * a[e];
        dgn += t.dl * (a[e] * s.inv + ctl_bias<false>(p, h, i));
      }
    }
    dsh = row_pair_sum(dsh, pair);
    s.dmarg = row_pair_sum(dmarg, pair);
    s.dmx = cnt > 0.f ? -dsh / cnt : 0.f;
    for (int c = 16 * part; c < p.PP; c += kChunkStep) {
      float a[16];
      tmem_ld16(ta_row + c, a);
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const int i = c + e;
        if (i >= p.P || softmax_logit(p, h, i, a[e], s.inv) != s.mx) continue;
        dot += ctl_gain<false>(p, h, i) * s.dmx * a[e];
        dgn += s.dmx * (a[e] * s.inv + ctl_bias<false>(p, h, i));
      }
    }
    s.dot_a = row_pair_sum(dot, pair);
    s.dgain = row_pair_sum(dgn, pair);
  }
  return s;
}

// Row statistics of the feature map; the kParts threads of a row each reduce
// their column chunks and combine through `pair` (kThreads floats of shared
// memory).  relu2: ss pass, then mass (and sum g u^2) pass.  softmax: ss
// pass, then one online pass for the max, the partition sum E and sum g e
// (each part rescales its running sums when its max grows; the parts are
// combined at the common max).  With kWithGrad, `grad16(c, g)` supplies the
// feature gradient of columns [c, c+16) and dphi = sum_j g_j phi_j, and the
// same pass forms the row totals that need dpre_j only through sums:
//   relu2   dpre_j = (g_j - dphi) 2 u_j / mass, so
//           dot_a = 2/mass (sum g u a - dphi sum u a), dthr = -2/mass (sum g u - dphi sum u);
//   softmax dpre_j = gain_j phi_j (g_j - dphi), phi_j = e_j / E, so
//           dot_a = (sum gain e g a - dphi sum gain e a) / E,
//           dgain = (sum e g sc - dphi sum e sc) / E
// (the softmax sums rescaled with E when the running max grows).
template <int KF, bool kWithGrad, class Grad>
__device__ __forceinline__ RowState row_stats(const FeatParams& p, uint32_t ta_row, int h, float* pair, Grad grad16) {
  constexpr int KIND = KF & kKindMask;
  constexpr bool kPlain = (KF & kPlainBit) != 0;
  if constexpr (KIND == kSoftmaxSparse) return row_stats_sparse<KF, kWithGrad>(p, ta_row, h, pair, grad16);
  const int part = my_part();
  RowState s{0.f, 0.f, -INFINITY, 0.f, 0.f, 0.f, 0.f};
  float ss = 0.f;
  if (p.PP == 4 * kChunkStep) {
    // the common width (256 features): all four chunks behind one wait
    float a4[4][16];
    tmem_ld16x4(ta_row + 16 * part, kChunkStep, a4);
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
      for (int e = 0; e < 16; ++e) ss += a4[k][e] * a4[k][e];
  } else {
    for (int c = 16 * part; c < p.PP; c += kChunkStep) {
      float a[16];
      tmem_ld16(ta_row + c, a);
#pragma unroll
      for (int e = 0; e < 16; ++e) ss += a[e] * a[e];
    }
  }
  ss = row_pair_sum(ss, pair);
  s.inv = rsqrtf(ss / static_cast<float>(p.P) + p.eps);
  if constexpr (KIND == kRelu2) {
    const float thr = ctl_thr<kPlain>(p, h);
    float M = 0.f, Sg = 0.f, Sgua = 0.f, Sua = 0.f, Sgu = 0.f, Su = 0.f;
    if constexpr (kPlain) {
      // u = relu(a * inv) over whole chunks, two columns per instruction
      const float2 inv2 = f2(s.inv, s.inv);
      float2 M2 = f2(0.f, 0.f), Sg2 = M2, Sgua2 = M2, Sua2 = M2, Sgu2 = M2, Su2 = M2;
      for (int c = 16 * part; c < p.PP; c += kChunkStep) {
        float a[16], g[16];
        tmem_ld16(ta_row + c, a);
        if (kWithGrad) grad16(c, g);
#pragma unroll
        for (int e = 0; e < 16; e += 2) {
          const float2 a2 = f2(a[e], a[e + 1]);
          const float2 u2 = relu2_u(a2, inv2);
          M2 = __ffma2_rn(u2, u2, M2);
          if (kWithGrad) {
            const float2 gu2 = __fmul2_rn(f2(g[e], g[e + 1]), u2);
            Sg2 = __ffma2_rn(gu2, u2, Sg2);
            Sgua2 = __ffma2_rn(gu2, a2, Sgua2);
            Sua2 = __ffma2_rn(u2, a2, Sua2);
            Sgu2 = __fadd2_rn(Sgu2, gu2);
            Su2 = __fadd2_rn(Su2, u2);
          }
        }
      }
      M = M2.x + M2.y;
      Sg = Sg2.x + Sg2.y;
      Sgua = Sgua2.x + Sgua2.y;
      Sua = Sua2.x + Sua2.y;
      Sgu = Sgu2.x + Sgu2.y;
      Su = Su2.x + Su2.y;
    } else
    for (int c = 16 * part; c < p.PP; c += kChunkStep) {
      float a[16], g[16];
      tmem_ld16(ta_row + c, a);
      if (kWithGrad) grad16(c, g);
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const int i = c + e;
        if (kPlain || i < p.P) {
          const float u = fmaxf(a[e] * s.inv + ctl_bias<kPlain>(p, h, i) - thr, 0.f);
          M += u * u;
          if (kWithGrad) {
            const float gu = g[e] * u;
            Sg += gu * u;
            Sgua += gu * a[e];
            Sua += u * a[e];
            Sgu += gu;
            Su += u;
          }
        }
      }
    }
    s.mass = row_pair_sum(M, pair);
    if (kWithGrad) {
      Sg = row_pair_sum(Sg, pair);
      Sgua = row_pair_sum(Sgua, pair);
      Sua = row_pair_sum(Sua, pair);
      Sgu = row_pair_sum(Sgu, pair);
      Su = row_pair_sum(Su, pair);
      if (s.mass > p.eps) {
        s.dphi = Sg / s.mass;
        const float k2 = 2.f / s.mass;
        s.dot_a = k2 * (Sgua - s.dphi * Sua);
        s.dthr = -k2 * (Sgu - s.dphi * Su);
      }
    }
  } else if constexpr (KIND == kSoftmax) {
    float m = -INFINITY, E = 0.f, Sg = 0.f, T1 = 0.f, T2 = 0.f, T3 = 0.f, T4 = 0.f;
    for (int c = 16 * part; c < p.PP; c += kChunkStep) {
      float a[16], g[16], l[16];
      tmem_ld16(ta_row + c, a);
      if (kWithGrad) grad16(c, g);
      float cm = -INFINITY;
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const int i = c + e;
        l[e] = (kPlain || i < p.P) ? ctl_gain<kPlain>(p, h, i) * (a[e] * s.inv + ctl_bias<kPlain>(p, h, i)) : -INFINITY;
        cm = fmaxf(cm, l[e]);
      }
      if (cm > m) {
        const float r = __expf(m - cm);
        E *= r;
        if (kWithGrad) {
          Sg *= r;
          T1 *= r;
          T2 *= r;
          T3 *= r;
          T4 *= r;
        }
        m = cm;
      }
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const int i = c + e;
        if (kPlain || i < p.P) {
          const float w = __expf(l[e] - m);
          E += w;
          if (kWithGrad) {
            const float gain = ctl_gain<kPlain>(p, h, i);
            const float sc = a[e] * s.inv + ctl_bias<kPlain>(p, h, i);
            const float gw = g[e] * w;
            Sg += gw;
            T1 += gain * gw * a[e];
            T2 += gain * w * a[e];
            T3 += gw * sc;
            T4 += w * sc;
          }
        }
      }
    }
    s.mx = row_pair_max(m, pair);
    const float r = __expf(m - s.mx);  // 0 for a part without columns (m = -inf)
    s.mass = row_pair_sum(E * r, pair);
    if (kWithGrad) {
      const float inv_E = 1.f / s.mass;
      s.dphi = row_pair_sum(Sg * r, pair) * inv_E;
      T1 = row_pair_sum(T1 * r, pair);
      T2 = row_pair_sum(T2 * r, pair);
      T3 = row_pair_sum(T3 * r, pair);
      T4 = row_pair_sum(T4 * r, pair);
      s.dot_a = (T1 - s.dphi * T2) * inv_E;
      s.dgain = (T3 - s.dphi * T4) * inv_E;
    }
  }
  return s;
}

// phi values for columns [c, c+16) of the (relu2 / softmax) feature row.
template <int KF>
__device__ __forceinline__ void phi_chunk(const FeatParams& p, const RowState& s, const float* a, int c, int h,
                                          float* out) {
  constexpr int KIND = KF & kKindMask;
  constexpr bool kPlain = (KF & kPlainBit) != 0;
  (void)kPlain;
  if constexpr (KIND == kRelu2 && kPlain) {
    const bool live = s.mass > p.eps;
    const float inv_mass = 1.f / fmaxf(s.mass, p.eps);
    const float2 inv2 = f2(s.inv, s.inv), im2 = f2(inv_mass, inv_mass);
    const float uniform = 1.f / static_cast<float>(p.m);
#pragma unroll
    for (int e = 0; e < 16; e += 2) {
      const float2 u2 = relu2_u(f2(a[e], a[e + 1]), inv2);
      const float2 v2 = __fmul2_rn(__fmul2_rn(u2, u2), im2);
      out[e] = live ? v2.x : uniform;
      out[e + 1] = live ? v2.y : uniform;
    }
  } else if constexpr (KIND == kRelu2) {
    const float thr = ctl_thr<kPlain>(p, h);
    const bool live = s.mass > p.eps;
    const float inv_mass = 1.f / fmaxf(s.mass, p.eps);
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const int i = c + e;
      const float u = fmaxf(a[e] * s.inv + ctl_bias<kPlain>(p, h, (kPlain || i < p.P) ? i : 0) - thr, 0.f);
      out[e] = (kPlain || i < p.P) ? (live ? u * u * inv_mass : 1.f / static_cast<float>(p.m)) : 0.f;
    }
  } else if constexpr (KIND == kSoftmaxSparse) {
    const float inv_E = 1.f / s.mass, inv_Z = 1.f / fmaxf(s.z, p.eps);
    const bool blend = p.sparse_mode == 3;
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const int i = c + e;
      float v = 0.f;
      if (i < p.P) {
        const float ex = expf(softmax_logit(p, h, i, a[e], s.inv) - s.mx);
        float gt, dgt;
        sparse_gate(p, softmax_logit(p, h, i, a[e], s.inv) - s.mx - s.lrho, gt, dgt);
        const float dense = ex * inv_E, sparse = ex * gt * inv_Z;
        v = blend ? dense + s.alpha * (sparse - dense) : sparse;
      }
      out[e] = v;
    }
  } else {
    const float inv_E = 1.f / s.mass;
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const int i = c + e;
      out[e] = (kPlain || i < p.P) ? __expf(ctl_gain<kPlain>(p, h, i) * (a[e] * s.inv + ctl_bias<kPlain>(p, h, i)) - s.mx) * inv_E : 0.f;
    }
  }
}

// ------------------------------------------------------------------ row prologue

// Rotation factors of the 8 channel pairs of columns [c, c+16) at sequence
// position t (zero-extended past rot): one vector load per table when the
// tables allow it.
struct Rot8 {
  float cs[8], sn[8];
};
__device__ __forceinline__ Rot8 load_rot8(const FeatParams& p, int t, int c) {
  Rot8 r;
  const int hr = p.rot >> 1;
  const size_t base = static_cast<size_t>(t) * hr + (c >> 1);
  if (c + 16 <= p.rot && (hr & 3) == 0) {
    const float4* pc = reinterpret_cast<const float4*>(p.rcos + base);
    const float4* ps = reinterpret_cast<const float4*>(p.rsin + base);
    const float4 c0 = __ldg(pc), c1 = __ldg(pc + 1), s0 = __ldg(ps), s1 = __ldg(ps + 1);
    const float cv[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    const float sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      r.cs[i] = cv[i];
      r.sn[i] = sv[i];
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const bool in = c + 2 * i < p.rot;
      r.cs[i] = in ? __ldg(p.rcos + base + i) : 1.f;
      r.sn[i] = in ? __ldg(p.rsin + base + i) : 0.f;
    }
  }
  return r;
}

// Adjacent-pair rotation of 16 consecutive channels [c, c+16) of the row, in
// f32 with separately rounded products as the reference's elementwise tensor
// ops round them (rope.py:69-70); channels past rot are left as they are.
// `inverse` applies the transpose (the backward of the rotation).
__device__ __forceinline__ void rotate16(const FeatParams& p, const Rot8& r, int c, float* f, bool inverse) {
#pragma unroll
  for (int e = 0; e < 16; e += 2) {
    if (c + e >= p.rot) break;
    const float cs = r.cs[e >> 1], sn = r.sn[e >> 1];
    const float x1 = f[e], x2 = f[e + 1];
    if (!inverse) {
      f[e] = __fsub_rn(__fmul_rn(x1, cs), __fmul_rn(x2, sn));
      f[e + 1] = __fadd_rn(__fmul_rn(x1, sn), __fmul_rn(x2, cs));
    } else {
      f[e] = __fadd_rn(__fmul_rn(x1, cs), __fmul_rn(x2, sn));
      f[e + 1] = __fsub_rn(__fmul_rn(x2, cs), __fmul_rn(x1, sn));
    }
  }
}

constexpr int kMaxRowChunks = 128 / kChunkStep;  // 16-column chunks per thread for d <= 128

// In place on the staged x tile: rotate each valid row, L2-normalize it
// (row / max(||row||, eps)) and round to bf16, so that the projection and the
// y0 residual see the reference's post-RoPE, post-norm rows.  `row_norm[r]`
// keeps the divisor of row r for the backward, negated when the eps clamp was
// active (then the norm passes no gradient).  Needs the tile complete and
// visible (after tiles_ready()); ends with the tile rewritten but no barrier.
__device__ void prepare_rows(const FeatParams& p, const Tile& tx, int t0, int rows, float* row_norm, float* pair) {
  const int row = my_row(), part = my_part();
  const bool valid = row < rows;
  const int t = p.pos0 + t0 + row;
  float v[kMaxRowChunks][16];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kMaxRowChunks; ++k) {
    const int c = 16 * part + kChunkStep * k;
    if (c >= p.dP) break;
    unpack8(tile_ld16(tx, row, c / 8), v[k]);
    unpack8(tile_ld16(tx, row, c / 8 + 1), v[k] + 8);
    if (valid && c < p.rot) rotate16(p, load_rot8(p, t, c), c, v[k], false);
#pragma unroll
    for (int e = 0; e < 16; ++e) ss = fmaf(v[k][e], v[k][e], ss);
  }
  float N = 1.f;
  if (p.l2norm) {
    ss = row_pair_sum(ss, pair);
    const float n = sqrtf(ss);
    N = fmaxf(n, p.neps);
    if (part == 0) row_norm[row] = n >= p.neps ? N : -N;
  }
  if (!valid) return;
#pragma unroll
  for (int k = 0; k < kMaxRowChunks; ++k) {
    const int c = 16 * part + kChunkStep * k;
    if (c >= p.dP) break;
    if (p.l2norm) {
#pragma unroll
      for (int e = 0; e < 16; ++e) v[k][e] = __fdiv_rn(v[k][e], N);
    }
    tile_st16(tx, row, c / 8, pack8(v[k]));
    tile_st16(tx, row, c / 8 + 1, pack8(v[k] + 8));
  }
}

// 16 bf16 values [c, c+16) of the row at `src` as floats (zero past width).
__device__ __forceinline__ void load_row16(const __nv_bfloat16* src, int c, int width, float* f) {
  const bool vec = ((reinterpret_cast<uintptr_t>(src + c) & 15) == 0) && c + 16 <= width;
  if (vec) {
    unpack8(__ldg(reinterpret_cast<const uint4*>(src + c)), f);
    unpack8(__ldg(reinterpret_cast<const uint4*>(src + c + 8)), f + 8);
  } else {
#pragma unroll
    for (int e = 0; e < 16; ++e) f[e] = c + e < width ? bf2f(src[c + e]) : 0.f;
  }
}

// 16 raw channels [c, c+16) of row t0 + row of selection `sel` (zero past d).
__device__ __forceinline__ void load_raw16(const FeatParams& p, int sel, int b, int h, int tok, int c, float* f) {
  load_row16(p.x[sel] + b * p.xs[sel][0] + h * p.xs[sel][1] + static_cast<long long>(tok) * p.xs[sel][2], c, p.d, f);
}

// Row-gradient epilogue of the backward.  TMEM columns [0, dP) at `t_dx` hold
// the gradient of the rows as the projection saw them (plus `addend`, f32
// [rows, d] row-major, when given).  With the fused prologue it is carried
// back through the normalization and the rotation to the raw rows.  Written
// as f32 rows of p.dx[sel] (contiguous) or bf16 rows of p.dxb[sel] (strided).
__device__ void store_row_grads(const FeatParams& p, uint32_t t_dx, int sel, int b, int h, int t0, int rows,
                                bool add_dy, size_t rowbase, const float* row_norm, float* pair) {
  const int row = my_row(), part = my_part(), quad = my_quad();
  const bool valid = row < rows;
  const int tok = t0 + row;
  const int t = p.pos0 + tok;
  // Global inputs first, so that their latencies overlap: the raw row and the
  // rotation factors (for the normalization backward) and the addend.
  float xh[kMaxRowChunks][16];
  Rot8 rot[kMaxRowChunks];
  float g[kMaxRowChunks][16];
#pragma unroll
  for (int k = 0; k < kMaxRowChunks; ++k) {
    const int c = 16 * part + kChunkStep * k;
    if (c >= p.dP) break;
    if (p.l2norm && valid) load_raw16(p, sel, b, h, tok, c, xh[k]);
    if (valid && c < p.rot) rot[k] = load_rot8(p, t, c);
    tmem_ld16(tmem_addr(t_dx, quad * 32, c), g[k]);
    if (add_dy && valid) {
      float dy[16];
      if (p.dyb != nullptr) {
        load_row16(p.dyb + b * p.dys[0] + h * p.dys[1] + static_cast<long long>(tok) * p.dys[2], c, p.d, dy);
      } else {
        const float* src = p.dy + (rowbase + row) * p.d;
#pragma unroll
        for (int e = 0; e < 16; ++e) dy[e] = c + e < p.d ? __ldg(src + c + e) : 0.f;
      }
#pragma unroll
      for (int e = 0; e < 16; ++e) g[k][e] += dy[e];
    }
  }
  if (p.l2norm) {
    // d raw = (g - xhat (xhat . g)) / N, or g / N where the eps clamp held.
    const float Ns = valid ? row_norm[row] : 1.f;
    const float invN = 1.f / fabsf(Ns);
    float dot = 0.f;
#pragma unroll
    for (int k = 0; k < kMaxRowChunks; ++k) {
      const int c = 16 * part + kChunkStep * k;
      if (c >= p.dP) break;
      if (valid) {
        if (c < p.rot) rotate16(p, rot[k], c, xh[k], false);
      } else {
#pragma unroll
        for (int e = 0; e < 16; ++e) xh[k][e] = 0.f;
      }
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        xh[k][e] *= invN;
        dot = fmaf(xh[k][e], g[k][e], dot);
      }
    }
    dot = row_pair_sum(dot, pair);
    const float proj = Ns > 0.f ? dot : 0.f;
#pragma unroll
    for (int k = 0; k < kMaxRowChunks; ++k) {
      const int c = 16 * part + kChunkStep * k;
      if (c >= p.dP) break;
#pragma unroll
      for (int e = 0; e < 16; ++e) g[k][e] = (g[k][e] - xh[k][e] * proj) * invN;
    }
  }
  if (!valid) return;
  const bool bf16 = p.dxb[sel] != nullptr;
#pragma unroll
  for (int k = 0; k < kMaxRowChunks; ++k) {
    const int c = 16 * part + kChunkStep * k;
    if (c >= p.dP) break;
    if (c < p.rot) rotate16(p, rot[k], c, g[k], true);
    if (bf16) {
      __nv_bfloat16* dst = p.dxb[sel] + b * p.dxs[sel][0] + h * p.dxs[sel][1] + static_cast<long long>(tok) * p.dxs[sel][2];
      if (((reinterpret_cast<uintptr_t>(dst + c) & 15) == 0) && c + 16 <= p.d) {
        *reinterpret_cast<uint4*>(dst + c) = pack8(g[k]);
        *reinterpret_cast<uint4*>(dst + c + 8) = pack8(g[k] + 8);
      } else {
        #pragma unroll
        for (int e = 0; e < 16; ++e)
          if (c + e < p.d) dst[c + e] = __float2bfloat16_rn(g[k][e]);
      }
    } else {
      float* dst = p.dx[sel] + ((static_cast<size_t>(b) * p.H + h) * p.T + tok) * p.d;
      #pragma unroll
      for (int e = 0; e < 16; ++e)
        if (c + e < p.d) dst[c + e] = g[k][e];
    }
  }
}

// ------------------------------------------------------------------ forward

__device__ __forceinline__ float tile_elem(const Tile& t, int r, int c) {
  unsigned short u;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(u) : "r"(t.saddr + tile_off(t, r, c)));
  return __bfloat162float(__ushort_as_bfloat16(u));
}

// phi of this thread's row and column chunks into the phi tile (bf16).
template <int KF>
__device__ __forceinline__ void phi_row_to_tile(const FeatParams& p, const RowState& st, uint32_t ta_row, int h,
                                                const Tile& tphi, bool zero_row, const SplineTable* spl,
                                                float* row32 = nullptr) {
  constexpr int KIND = KF & kKindMask;
  constexpr bool kPlain = (KF & kPlainBit) != 0;
  (void)kPlain;
  const int row = my_row(), part = my_part();
  if constexpr (KIND == kBspline) {
    const float sc = ctl_scale(p, h);
    const float invP = 1.f / static_cast<float>(p.P);
    // This thread's projections pj = kParts * i + part, gathered first so that
    // the basis evaluation below is one compact loop (one copy of its code).
    float a_own[kMaxSplineOwn];
#pragma unroll
    for (int i = 0; i < kMaxSplineOwn; ++i) a_own[i] = 0.f;
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
      const int c = 16 * cc;
      if (c >= p.PP) break;
      float a[16];
      tmem_ld16(ta_row + c, a);
#pragma unroll
      for (int e = 0; e < 16; ++e)
        if ((e % kParts) == part) a_own[(c + e) / kParts] = a[e];
    }
#pragma unroll 1
    for (int i = 0; i < kMaxSplineOwn; ++i) {
      const int pj = kParts * i + part;
      if (pj >= p.P) break;
      float val[4], der[4];
      int first;
      bool inside;
      bspline_local(a_own[i] * st.inv * sc, p.nb, p.bound, *spl, val, der, first, inside);
      for (int ii = 0; ii < p.nb; ii += 8) {
        float f[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const int w = ii + q - first;
          f[q] = (!zero_row && w >= 0 && w < 4) ? pick4(val, w) * invP : 0.f;
        }
        tile_st16(tphi, row, (pj * p.nb + ii) / 8, pack8(f));
        if (row32 != nullptr && !zero_row) {
          float4* dst = reinterpret_cast<float4*>(row32 + pj * p.nb + ii);
          dst[0] = make_float4(f[0], f[1], f[2], f[3]);
          dst[1] = make_float4(f[4], f[5], f[6], f[7]);
        }
      }
    }
  } else {
    for (int c = 16 * part; c < p.PP; c += kChunkStep) {
      float a[16], f[16];
      tmem_ld16(ta_row + c, a);
      phi_chunk<KF>(p, st, a, c, h, f);
      if (zero_row) {
#pragma unroll
        for (int e = 0; e < 16; ++e) f[e] = 0.f;
      }
      tile_st16(tphi, row, c / 8, pack8(f));
      tile_st16(tphi, row, c / 8 + 1, pack8(f + 8));
      if (row32 != nullptr && !zero_row) {
        #pragma unroll
        for (int e = 0; e < 16; ++e)
          if (c + e < p.m) row32[c + e] = f[e];
      }
    }
  }
}

// Persistent over tiles: CTA (c, h) owns head h's tiles c, c + G, c + 2G, ...
// of the (b, sel, n) tiles of that head (G = gridDim.x), so W1 and W2 are
// staged once, TMEM and the barrier are set up once, and the next tile's rows
// are copied in (cp.async, a second x buffer) while this tile computes.
__device__ __forceinline__ void feature_tile_coords(const FeatParams& p, int i, int NT, int& b, int& sel, int& n) {
  n = i % NT;
  const int rest = i / NT;
  sel = p.sel0 + rest % p.nsel;
  b = rest / p.nsel;
}

template <int KF>
__global__ void __launch_bounds__(kThreads, 1) feature_fwd_kernel(FeatParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint64_t bar;
  __shared__ uint32_t tmem_base;
  __shared__ SplineTable spl_table;
  if constexpr ((KF & kKindMask) == kBspline) build_spline_table(spl_table, p.nb, p.bound);
  __shared__ float pair[kThreads];
  __shared__ float row_norm[kTile];
  const int h = blockIdx.y;
  const int row = my_row(), quad = my_quad();
  const int warp = threadIdx.x >> 5;
  const int NT = (p.T + kTile - 1) / kTile;
  const int ntiles = p.B * p.nsel * NT;
  const bool any_decode = p.sel0 + p.nsel > 1 && p.y0 != nullptr && p.W2 != nullptr;

  const uint32_t base = smem_u32(smem);
  FeatTiles tl;
  Tile xbuf[2];
  xbuf[0] = Tile{base, kTile, p.dP};
  xbuf[1] = Tile{xbuf[0].saddr + kTile * p.dP * 2, kTile, p.dP};
  tl.w1 = Tile{xbuf[1].saddr + kTile * p.dP * 2, p.PP, p.dP};
  tl.phi = Tile{tl.w1.saddr + p.PP * p.dP * 2, kTile, p.mP};
  tl.w2 = Tile{tl.phi.saddr + kTile * p.mP * 2, p.dP, p.mP};
  float* stage = reinterpret_cast<float*>(smem + (tl.w2.saddr + p.dP * p.mP * 2 - base));

  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(&tmem_base, 512);
  auto load_x = [&](int i, const Tile& dst) {
    int b, sel, n;
    feature_tile_coords(p, i, NT, b, sel, n);
    const int t0 = n * kTile;
    const __nv_bfloat16* xp =
        p.x[sel] + b * p.xs[sel][0] + h * p.xs[sel][1] + static_cast<long long>(t0) * p.xs[sel][2];
    load_tile(dst, xp, p.xs[sel][2], min(kTile, p.T - t0), p.d);
  };
  load_tile(tl.w1, p.W1 + static_cast<size_t>(h) * p.P * p.d, p.d, p.P, p.d);
  if (any_decode) load_tile(tl.w2, p.W2 + static_cast<size_t>(h) * p.d * p.m, p.m, p.d, p.m);
  if (static_cast<int>(blockIdx.x) < ntiles) load_x(blockIdx.x, xbuf[0]);
  tiles_ready();
  MmaCtx ctx{&bar, tmem_base, 0u, true};
  const uint32_t t_a = ctx.tmem, t_y = ctx.tmem + 256;
  const uint32_t ta_row = tmem_addr(t_a, quad * 32, 0);

  int k = 0;
  for (int i = blockIdx.x; i < ntiles; i += gridDim.x, ++k) {
    int b, sel, n;
    feature_tile_coords(p, i, NT, b, sel, n);
    const int t0 = n * kTile;
    const int rows = min(kTile, p.T - t0);
    const bool decode = sel == 1 && any_decode;
    tl.x = xbuf[k & 1];
    // the next tile's rows stream in while this one computes
    if (i + static_cast<int>(gridDim.x) < ntiles) load_x(i + gridDim.x, xbuf[(k + 1) & 1]);
    cp_async_commit();
    cp_async_wait_group<1>();
    __syncthreads();
    if (p.rot > 0 || p.l2norm) prepare_rows(p, tl.x, t0, rows, row_norm, pair);
    ctx.run_keep_newest([&] { gemm_issue(t_a, kmajor(tl.x), kmajor(tl.w1), p.PP, p.dP, false); });

    const RowState st = row_stats<KF, false>(p, ta_row, h, pair, NoGrad{});
    // Rows past the sequence end get zero features, so the decode below and
    // the stored tile are exact zeros there.
    float* row32 = (sel == 1 && p.phi_q32 != nullptr && row < rows)
                      ? p.phi_q32 + ((static_cast<size_t>(b) * p.H + h) * p.T + t0 + row) * p.m : nullptr;
    phi_row_to_tile<KF>(p, st, ta_row, h, tl.phi, row >= rows, &spl_table, row32);
    __syncthreads();
    __nv_bfloat16* out = p.phi[sel] + ((static_cast<size_t>(b) * p.H + h) * p.T + t0) * p.m;
    store_tile(tl.phi, out, p.m, rows, p.m);
    if (decode) {
      ctx.run_keep_newest([&] { gemm_issue(t_y, kmajor(tl.phi), kmajor(tl.w2), p.dP, p.mP, false); });
      float* y0 = p.y0 + ((static_cast<size_t>(b) * p.H + h) * p.T + t0) * p.d;
      const Tile tx = tl.x;
      store_rows(t_y, 0, p.dP, p.d, rows, y0, p.d, false, stage,
                 [&](int r, int col, float v) { return col < p.d ? v + tile_elem(tx, r, col) : v; });
    }
    // everything of this tile (x, phi, stage, TMEM) is consumed before the
    // next iteration refills it
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  }
  cp_async_wait_all();
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem_base, 512);
}

// ------------------------------------------------------------------ backward

template <int KF>
__global__ void __launch_bounds__(kThreads, 1) feature_bwd_kernel(FeatParams p) {
  constexpr int KIND = KF & kKindMask;
  constexpr bool kPlain = (KF & kPlainBit) != 0;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint64_t bar;
  __shared__ uint32_t tmem_base;
  __shared__ SplineTable spl_table;
  if constexpr (KIND == kBspline) build_spline_table(spl_table, p.nb, p.bound);
  __shared__ float red[32];
  __shared__ float pair[kThreads];
  __shared__ float row_norm[kTile];
  const int n = blockIdx.x, h = blockIdx.y;
  const int b = blockIdx.z / p.nsel, sel = p.sel0 + blockIdx.z % p.nsel;
  const int row = my_row(), part = my_part(), quad = my_quad();
  const int warp = threadIdx.x >> 5;
  const int t0 = n * kTile;
  const int rows = min(kTile, p.T - t0);
  const bool valid = row < rows;
  const bool decode = sel == 1 && (p.dy != nullptr || p.dyb != nullptr) && p.W2 != nullptr;
  constexpr bool spline = KIND == kBspline;

  const uint32_t base = smem_u32(smem);
  FeatTiles tl;
  tl.x = Tile{base, kTile, p.dP};
  tl.w1 = Tile{tl.x.saddr + kTile * p.dP * 2, p.PP, p.dP};
  tl.da = Tile{tl.w1.saddr + p.PP * p.dP * 2, kTile, p.PM};
  tl.phi = Tile{tl.da.saddr + kTile * p.PM * 2, kTile, p.mM};
  tl.dy = Tile{tl.phi.saddr + kTile * p.mM * 2, kTile, p.dP};
  tl.w2 = Tile{tl.dy.saddr + kTile * p.dP * 2, p.dP, p.mP};
  // dphi: in place of dA for relu2 / softmax (column j of both is feature j,
  // and each thread overwrites one of its own chunks only after reading it);
  // separate for B-splines, whose dphi columns are (projection, basis) pairs.
  const Tile tdphi = spline ? Tile{tl.w2.saddr + p.dP * p.mP * 2, kTile, p.mP} : Tile{tl.da.saddr, kTile, p.PM};

  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(&tmem_base, 512);
  const size_t rowbase = (static_cast<size_t>(b) * p.H + h) * p.T + t0;
  const __nv_bfloat16* xp = p.x[sel] + b * p.xs[sel][0] + h * p.xs[sel][1] + static_cast<long long>(t0) * p.xs[sel][2];
  load_tile(tl.x, xp, p.xs[sel][2], rows, p.d);
  load_tile(tl.w1, p.W1 + static_cast<size_t>(h) * p.P * p.d, p.d, p.P, p.d);
  const void* dphi_src = p.dphi_bf16
      ? static_cast<const void*>(static_cast<const __nv_bfloat16*>(p.dphi[sel]) + rowbase * p.m)
      : static_cast<const void*>(static_cast<const float*>(p.dphi[sel]) + rowbase * p.m);
  load_tile_any(tdphi, dphi_src, p.m, rows, p.m, p.dphi_bf16 != 0);
  // The decode gradient dW2 += phi(q)^T dy rebuilds phi(q) from the TMEM
  // pre-activations in the sweep below: measured faster than loading the
  // forward's bf16 tile (0.05 ms of 1.46 per config-2 step).
  if (decode) {
    load_tile(tl.w2, p.W2 + static_cast<size_t>(h) * p.d * p.m, p.m, p.d, p.m);
    if (p.dyb != nullptr) {
      load_tile(tl.dy, p.dyb + b * p.dys[0] + h * p.dys[1] + static_cast<long long>(t0) * p.dys[2], p.dys[2], rows,
                p.d);
    } else {
      load_tile_any(tl.dy, p.dy + rowbase * p.d, p.d, rows, p.d, false);
    }
  }
  // dA columns no sweep writes must be zero (the dW1 product reads PM of them).
  for (int j = (spline ? 0 : p.PP / 8) + part; j < p.PM / 8; j += kParts)
    tile_st16(tl.da, row, j, make_uint4(0, 0, 0, 0));
  tiles_ready();
  if (p.rot > 0 || p.l2norm) prepare_rows(p, tl.x, t0, rows, row_norm, pair);
  MmaCtx ctx{&bar, tmem_base, 0u, true};
  const uint32_t t_a = ctx.tmem, t_hi = ctx.tmem + 256;
  ctx.run([&] {
    gemm_issue(t_a, kmajor(tl.x), kmajor(tl.w1), p.PP, p.dP, false);
    if (decode) gemm_issue(t_hi, kmajor(tl.dy), mnmajor(tl.w2), p.mP, p.dP, false);
  });

  const uint32_t ta_row = tmem_addr(t_a, quad * 32, 0);
  const uint32_t tb_row = tmem_addr(t_hi, quad * 32, 0);
  // Total gradient of 16 feature columns [c, c+16) of this row: staged dphi
  // plus the slow-decode contribution dy W2 (TMEM).
  auto grad16 = [&](int c, float* g) {
    unpack8(tile_ld16(tdphi, row, c / 8), g);
    unpack8(tile_ld16(tdphi, row, c / 8 + 1), g + 8);
    if (decode) {
      float dhi[16];
      tmem_ld16(tb_row + c, dhi);
#pragma unroll
      for (int e = 0; e < 16; ++e) g[e] += dhi[e];
    }
  };

  const RowState st = spline ? row_stats<KF, false>(p, ta_row, h, pair, NoGrad{})
                             : row_stats<KF, true>(p, ta_row, h, pair, grad16);
  const float dot_phi = st.dphi;  // sum_j g_j phi_j (relu2 / softmax Jacobians)
  // dpre for columns [c, c+16) (projection index for B-splines).
  auto dpre_chunk = [&](int c, const float* a, float* dp) {
    if constexpr (KIND == kRelu2) {
      float g[16];
      grad16(c, g);
      const float thr = ctl_thr<kPlain>(p, h);
      const bool live = st.mass > p.eps;
      const float inv_mass = 1.f / fmaxf(st.mass, p.eps);
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const int i = c + e;
        float d = 0.f;
        if ((kPlain || i < p.P) && live) {
          const float u = fmaxf(a[e] * st.inv + ctl_bias<kPlain>(p, h, i) - thr, 0.f);
          d = (g[e] - dot_phi) * inv_mass * 2.f * u;
        }
        dp[e] = d;
      }
    } else if constexpr (KIND == kSoftmax) {
      float g[16];
      grad16(c, g);
      const float inv_E = 1.f / st.mass;
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const int i = c + e;
        float d = 0.f;
        if (kPlain || i < p.P) {
          const float gain = ctl_gain<kPlain>(p, h, i);
          const float sc = a[e] * st.inv + ctl_bias<kPlain>(p, h, i);
          const float ph = __expf(gain * sc - st.mx) * inv_E;
          d = gain * ph * (g[e] - dot_phi);
        }
        dp[e] = d;
      }
    } else if constexpr (KIND == kSoftmaxSparse) {
      float g[16];
      grad16(c, g);
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const int i = c + e;
        float d = 0.f;
        if (i < p.P) {
          const float l = softmax_logit(p, h, i, a[e], st.inv);
          const float dl = sparse_terms(p, st, g[e], l).dl + (l == st.mx ? st.dmx : 0.f);
          d = ctl_gain<false>(p, h, i) * dl;
        }
        dp[e] = d;
      }
    } else {
      // B-splines run their own sweep (below).
#pragma unroll
      for (int e = 0; e < 16; ++e) dp[e] = 0.f;
    }
  };

  float dot_a = 0.f, dthr = 0.f, dscale = 0.f, dgain_head = 0.f, drho = 0.f, dalpha = 0.f;
  if constexpr (spline) {
    // B-splines: this thread's projections pj = kParts * i + part.  dpre of a
    // projection is sc * sum over the four live basis functions of
    // g(pj, basis) * basis' / P (zero where the coordinate was clamped).
    const float sc = ctl_scale(p, h);
    const float invP = 1.f / static_cast<float>(p.P);
    float a_own[kMaxSplineOwn], dp_own[kMaxSplineOwn];
#pragma unroll
    for (int i = 0; i < kMaxSplineOwn; ++i) a_own[i] = dp_own[i] = 0.f;
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
      const int c = 16 * cc;
      if (c >= p.PP) break;
      float a[16];
      tmem_ld16(ta_row + c, a);
#pragma unroll
      for (int e = 0; e < 16; ++e)
        if ((e % kParts) == part) a_own[(c + e) / kParts] = a[e];
    }
#pragma unroll 1
    for (int i = 0; i < kMaxSplineOwn; ++i) {
      const int pj = kParts * i + part;
      if (pj >= p.P) break;
      float val[4], der[4];
      int first;
      bool inside;
      bspline_local(a_own[i] * st.inv * sc, p.nb, p.bound, spl_table, val, der, first, inside);
      float g[16];
      grad16(pj * p.nb, g);   // basis functions 0..15 of projection pj (nb <= 16)
      float dc = 0.f;
#pragma unroll
      for (int q = 0; q < 16; ++q) {
        const int w = q - first;
        if (w >= 0 && w < 4) dc += g[q] * pick4(der, w) * invP;
      }
      const float d = inside ? dc * sc : 0.f;
      dp_own[i] = d;
      dot_a += d * a_own[i];
      dscale += d * a_own[i] * st.inv / sc;
    }
    dot_a = row_pair_sum(dot_a, pair);
    if (!valid) dot_a = dscale = 0.f;
    if (decode) phi_row_to_tile<KF>(p, st, ta_row, h, tl.phi, !valid, &spl_table);
    const float inv3 = st.inv * st.inv * st.inv / static_cast<float>(p.P);
#pragma unroll
    for (int i = 0; i < kMaxSplineOwn; ++i) {
      const int pj = kParts * i + part;
      if (pj >= p.P) break;
      const float da = valid ? st.inv * dp_own[i] - a_own[i] * inv3 * dot_a : 0.f;
      const __nv_bfloat16 v = __float2bfloat16_rn(da);
      asm volatile("st.shared.u16 [%0], %1;" ::"r"(tl.da.saddr + tile_off(tl.da, row, pj)),
                   "h"(__bfloat16_as_ushort(v))
                   : "memory");
    }
  } else {
    // The statistics pass formed dot_a = sum_j dpre_j a_j (RMSNorm backward)
    // and the per-head control gradients as row totals (counted once per row).
    dot_a = valid ? st.dot_a : 0.f;
    if (valid && part == 0) {
      dthr = st.dthr;
      dgain_head = st.dgain;
      if constexpr (KIND == kSoftmaxSparse) {
        // margin = shifted - log clamp(rho, eps, 1 - eps)
        const float rho = __ldg(p.rho + h);
        drho = rho >= p.eps && rho <= 1.f - p.eps ? -st.dmarg / rho : 0.f;
        dalpha = p.sparse_mode == 3 ? st.Ss - st.Sd : 0.f;
      }
    }
    // One sweep: (phi -> tile for dW2), dA = inv * dpre - a *
    // inv^3 * dot_a / P, and the per-feature control gradients.
    if (decode) phi_row_to_tile<KF>(p, st, ta_row, h, tl.phi, !valid, &spl_table);
    const float inv3 = st.inv * st.inv * st.inv / static_cast<float>(p.P);
    const bool dbias = p.bias != nullptr && p.dbias != nullptr && valid;
    const bool dgain_feat = (KIND == kSoftmax || KIND == kSoftmaxSparse) && p.gain_mode == 2 && valid;
    if constexpr (KIND == kRelu2 && kPlain) {
      // dpre = (g - dphi) (2 / mass) u (live rows), two columns per instruction
      const bool live = st.mass > p.eps && valid;
      const float k2 = 2.f / fmaxf(st.mass, p.eps);
      const float2 inv2 = f2(st.inv, st.inv), k22 = f2(k2, k2), mdphi = f2(-dot_phi, -dot_phi);
      const float2 c3 = f2(inv3 * dot_a, inv3 * dot_a);
      for (int c = 16 * part; c < p.PP; c += kChunkStep) {
        float a[16], g[16], da[16];
        tmem_ld16(ta_row + c, a);
        grad16(c, g);
#pragma unroll
        for (int e = 0; e < 16; e += 2) {
          const float2 a2 = f2(a[e], a[e + 1]);
          const float2 u2 = relu2_u(a2, inv2);
          const float2 dp2 = __fmul2_rn(__fmul2_rn(__fadd2_rn(f2(g[e], g[e + 1]), mdphi), k22), u2);
          const float2 x2 = __fmul2_rn(a2, c3);
          const float2 da2 = __ffma2_rn(inv2, live ? dp2 : f2(0.f, 0.f), f2(-x2.x, -x2.y));
          da[e] = valid ? da2.x : 0.f;
          da[e + 1] = valid ? da2.y : 0.f;
        }
        tile_st16(tl.da, row, c / 8, pack8(da));
        tile_st16(tl.da, row, c / 8 + 1, pack8(da + 8));
      }
    } else
    for (int c = 16 * part; c < p.PP; c += kChunkStep) {
      float a[16], dp[16], da[16];
      tmem_ld16(ta_row + c, a);
      dpre_chunk(c, a, dp);
  #pragma unroll
      for (int e = 0; e < 16; ++e) da[e] = valid ? st.inv * dp[e] - a[e] * inv3 * dot_a : 0.f;
      tile_st16(tl.da, row, c / 8, pack8(da));
      tile_st16(tl.da, row, c / 8 + 1, pack8(da + 8));
      if (dbias || dgain_feat) {
        #pragma unroll
        for (int e = 0; e < 16; ++e) {
          if (c + e >= p.P) break;
          if (dbias) atomicAdd(p.dbias + h * p.m + c + e, dp[e]);
          if (dgain_feat) {
            const float sc = a[e] * st.inv + ctl_bias<kPlain>(p, h, c + e);
            atomicAdd(p.dgain + h * p.m + c + e, dp[e] * sc / ctl_gain<kPlain>(p, h, c + e));
          }
        }
      }
    }
  }
  {
    const float s1 = block_sum(dthr, red);
    const float s2 = block_sum(dscale, red);
    const float s3 = block_sum(dgain_head, red);
    float s4 = 0.f, s5 = 0.f;
    if constexpr (KIND == kSoftmaxSparse) {
      s4 = block_sum(drho, red);
      s5 = block_sum(dalpha, red);
    }
    if (threadIdx.x == 0) {
      if (KIND == kRelu2 && p.thr && p.dthr) atomicAdd(p.dthr + h, s1);
      if (spline && p.scale && p.dscale) atomicAdd(p.dscale + h, s2);
      if ((KIND == kSoftmax || KIND == kSoftmaxSparse) && p.gain_mode == 1 && p.dgain) atomicAdd(p.dgain + h, s3);
      if (KIND == kSoftmaxSparse && p.drho) atomicAdd(p.drho + h, s4);
      if (KIND == kSoftmaxSparse && p.dalpha && p.sparse_mode == 3) atomicAdd(p.dalpha + h, s5);
    }
  }

  // dx = dA W1 (+ dy for q); dW1 += dA^T x; dW2^T += phi^T dy.
  const int pblocks = p.PM / kTile, mblocks = p.mM / kTile;
  ctx.run([&] {
    gemm_issue(t_hi, kmajor(tl.da), mnmajor(tl.w1), p.dP, p.PP, false);
    for (int mb = 0; mb < pblocks; ++mb)
      gemm_issue(t_a + mb * p.dP, mnmajor(tl.da, 0, mb * kTile), mnmajor(tl.x), p.dP, kTile, false);
    if (decode)
      for (int mb = 0; mb < mblocks; ++mb)
        gemm_issue(t_a + (pblocks + mb) * p.dP, mnmajor(tl.phi, 0, mb * kTile), mnmajor(tl.dy), p.dP, kTile,
                   false);
  });
  store_row_grads(p, t_hi, sel, b, h, t0, rows, decode, rowbase, row_norm, pair);
  for (int mb = 0; mb < pblocks; ++mb) {
    const int prj = mb * kTile + row;
    for (int c = 16 * part; c < p.dP; c += kChunkStep) {
      float v[16];
      tmem_ld16(tmem_addr(t_a + mb * p.dP, quad * 32, c), v);
      if (prj < p.P && p.dW1) {
        float* wrow = p.dW1 + (static_cast<size_t>(h) * p.P + prj) * p.d;
        #pragma unroll
        for (int e = 0; e < 16; e += 4) {
          if (c + e >= p.d) break;
          if (c + e + 4 <= p.d && (p.d & 3) == 0) {
            atomicAdd(reinterpret_cast<float4*>(wrow + c + e), make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]));
          } else {
            #pragma unroll
            for (int q = 0; q < 4; ++q)
              if (c + e + q < p.d) atomicAdd(wrow + c + e + q, v[e + q]);
          }
        }
      }
    }
  }
  if (decode) {
    for (int mb = 0; mb < mblocks; ++mb) {
      const int fi = mb * kTile + row;
      for (int c = 16 * part; c < p.dP; c += kChunkStep) {
        float v[16];
        tmem_ld16(tmem_addr(t_a + (pblocks + mb) * p.dP, quad * 32, c), v);
        if (fi < p.m && p.dW2) {
          if (p.dW2_t && (p.d & 3) == 0) {
            // [H, m, d]: this row's d values are contiguous
            float* wrow = p.dW2 + (static_cast<size_t>(h) * p.m + fi) * p.d;
            #pragma unroll
            for (int e = 0; e < 16; e += 4)
              if (c + e < p.d)
              atomicAdd(reinterpret_cast<float4*>(wrow + c + e), make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]));
          } else if (p.dW2_t) {
            #pragma unroll
            for (int e = 0; e < 16; ++e)
              if (c + e < p.d)
              atomicAdd(p.dW2 + (static_cast<size_t>(h) * p.m + fi) * p.d + c + e, v[e]);
          } else {
            #pragma unroll
            for (int e = 0; e < 16; ++e)
              if (c + e < p.d)
              atomicAdd(p.dW2 + (static_cast<size_t>(h) * p.d + c + e) * p.m + fi, v[e]);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem_base, 512);
}

// ------------------------------------------------------------------ host launch

size_t feature_fwd_smem(const FeatParams& p) {
  return static_cast<size_t>(2 * kTile * p.dP + p.PP * p.dP + kTile * p.mP + p.dP * p.mP) * 2 + kStageFloats * 4;
}

// CTAs per head of the persistent kernels: about one CTA per SM in all.
static int persistent_ctas_per_head(const FeatParams& p, int ntiles) {
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = 148;
  }
  const int g = sms / p.H;
  return max(1, min(ntiles, g));
}
size_t feature_bwd_smem(const FeatParams& p) {
  size_t bytes = static_cast<size_t>(kTile * p.dP + p.PP * p.dP + kTile * p.PM + kTile * p.mM + kTile * p.dP +
                                     p.dP * p.mP) * 2;
  if (p.kind == kBspline) bytes += static_cast<size_t>(kTile) * p.mP * 2;
  return bytes;
}

// One instantiation per feature kind: the kind decides the per-element code
// of every sweep, and specialising keeps each kind's locals in registers.
template <int KF>
static int launch_feature_fwd_kind(const FeatParams& p, cudaStream_t s) {
  const size_t sm = feature_fwd_smem(p);
  cudaFuncSetAttribute(feature_fwd_kernel<KF>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(sm));
  const int NT = ceil_div(p.T, kTile);
  const int G = persistent_ctas_per_head(p, p.B * p.nsel * NT);
  feature_fwd_kernel<KF><<<dim3(G, p.H), kThreads, sm, s>>>(p);
  return check_launch("feature_fwd_kernel");
}

template <int KF>
static int launch_feature_bwd_kind(const FeatParams& p, cudaStream_t s) {
  const size_t sm = feature_bwd_smem(p);
  cudaFuncSetAttribute(feature_bwd_kernel<KF>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(sm));
  const int NT = ceil_div(p.T, kTile);
  feature_bwd_kernel<KF><<<dim3(NT, p.H, p.B * p.nsel), kThreads, sm, s>>>(p);
  return check_launch("feature_bwd_kernel");
}

// A relu2 / softmax map without per-feature or per-head controls over whole
// column chunks runs the plain instantiation.
static bool plain_map(const FeatParams& p) {
  return p.kind != kBspline && p.sparse_mode == 0 && p.bias == nullptr && p.thr == nullptr && p.gain_mode == 0 && p.P == p.PP;
}

int launch_feature_fwd(const FeatParams& p, cudaStream_t s) {
  const bool plain = plain_map(p);
  switch (p.kind) {
    case kRelu2: return plain ? launch_feature_fwd_kind<kRelu2 | kPlainBit>(p, s) : launch_feature_fwd_kind<kRelu2>(p, s);
    case kSoftmax:
      if (p.sparse_mode) return launch_feature_fwd_kind<kSoftmaxSparse>(p, s);
      return plain ? launch_feature_fwd_kind<kSoftmax | kPlainBit>(p, s) : launch_feature_fwd_kind<kSoftmax>(p, s);
    default: return launch_feature_fwd_kind<kBspline>(p, s);
  }
}

int launch_feature_bwd(const FeatParams& p, cudaStream_t s) {
  const bool plain = plain_map(p);
  switch (p.kind) {
    case kRelu2: return plain ? launch_feature_bwd_kind<kRelu2 | kPlainBit>(p, s) : launch_feature_bwd_kind<kRelu2>(p, s);
    case kSoftmax:
      if (p.sparse_mode) return launch_feature_bwd_kind<kSoftmaxSparse>(p, s);
      return plain ? launch_feature_bwd_kind<kSoftmax | kPlainBit>(p, s) : launch_feature_bwd_kind<kSoftmax>(p, s);
    default: return launch_feature_bwd_kind<kBspline>(p, s);
  }
}

}  // namespace ts
