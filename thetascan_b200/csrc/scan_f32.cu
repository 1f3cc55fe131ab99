// Float32 streams: the multi-view scan on the CUDA cores at float32 accuracy.
//
// bf16 (2^-9) or tf32 (2^-11) tensor-core operands cannot meet the float32
// parity bound of the reference's fp32 configuration (rel-err 1e-5 against
// scan_chunk.linattn_views in float32, src/thetascan/_core/ops/
// scan_chunk.py:246-339), so f32 streams take this path: every product and
// every sum is an f32 FMA.  The tile algebra is the one of the tensor-core
// kernels.  For a tile of `len` tokens, local rows i, j, and a retention with
// log-retention la (0 for the plain sum), with e(x) = exp(la x):
//   intra weight w(i,j) = e(i-j) (j <= i), carry c(i) = e(i+1),
//   key weight u(j) = e(len-1-j), closing C = e(len);
//   out_i  = sum_{j<=i} w (q_i.k_j) v_j + c(i) q_i S_in
//   S_next = C S_in + sum_j u(j) k_j^T v_j
// Forward: (1) every tile's local update sum_j u k_j^T v_j, all tiles at once;
// (2) the exclusive prefix over tiles, per state element, in place; (3) every
// tile's outputs.  Backward, with G the gradient of the state leaving a tile:
// (1) every tile's local read gradient sum_i c(i) q_i^T dout_i; (2) the
// reverse exclusive prefix G(n-1) = local(n) + C G(n), with the closing
// term of d la; (3) per tile
//   ds  = sum_r w_r o (dout_r v^T)                 (causal)
//   dq_i = sum_j ds_ij k_j + sum_r c_r(i) S_in,r dout_r,i
//   dk_j = sum_i ds_ij q_i + sum_r u_r(j) G_r v_j
//   dv_j = sum_r [sum_{i>=j} w_r (q_i.k_j) dout_r,i + u_r(j) k_j G_r]
//   d la_r = sum (i-j) w s g + sum (i+1) c q_i.(S_in dout_i) + sum (len-1-j) u k_j.(G v_j)
//            + (prefix) sum_n len C <G(n), S_in(n)>.
// A per-token retention stream (the [B,H,T,1] decay of scan_chunk.py:122-155)
// replaces e(x) by the tile's cumulative log phases l_i = sum_{s<=i} la_s
// (f32, from the tile's first token): w(i,j) = exp(l_i - l_j), c(i) =
// exp(l_i), u(j) = exp(l_last - l_j), C = exp(l_last), every exponent <= 0.
// Its gradient is per token: d la_t = sum_{i>=t} dl_i within the tile, with
// dl_i collecting +row sums and -column sums of the intra terms, the carry
// term of row i, -/+ the key-weight terms of row j and the last row, and the
// tile's closing term C_n <G(n), S_in(n)> on the last row.
// Shared-memory tiles have odd leading dimensions, so that the row-strided
// reads of every loop fall in distinct banks.  The reference's fp32 case
// (B=2, H=4, T=512, d_k=64, payload 65) is a few hundred thousand FMAs per
// tile: latency-bound small work, not a roofline kernel.
#include "common.cuh"
#include "scan_f32.cuh"

namespace ts {

namespace {

constexpr int kF32Threads = 256;

__host__ __device__ __forceinline__ int odd_ld(int x) { return x | 1; }

__device__ __forceinline__ size_t f32_state_offset(const ScanF32Params& p, int bh, int n, int r) {
  return ((static_cast<size_t>(bh) * p.NT + n) * p.R + r) * static_cast<size_t>(p.Dk) * p.Dv;
}

// dst[i][c] (leading dimension ld) for i < TL, c < cols: the stream row
// src[i] for c < width, `fill` for width <= c < cols; zero for i >= rows.
__device__ void load_tile_f32(float* dst, int ld, const float* src, long long rs, int rows, int TL, int width,
                              int cols, float fill) {
  for (int e = threadIdx.x; e < TL * cols; e += blockDim.x) {
    const int i = e / cols, c = e - (e / cols) * cols;
    float x = 0.f;
    if (i < rows) x = c < width ? __ldg(src + i * rs + c) : fill;
    dst[i * ld + c] = x;
  }
}

// Weights of one retention over one tile, from a shared-memory table `tab`
// of TL + 1 floats: ex[x] = exp(la x) for a static retention (all ones for
// the plain sum), or the cumulative log phases l_i of a per-token stream.
struct TileWeights {
  const float* tab;
  bool stream;
  int rows;
  __device__ __forceinline__ float w(int i, int j) const { return stream ? expf(tab[i] - tab[j]) : tab[i - j]; }
  __device__ __forceinline__ float c(int i) const { return stream ? expf(tab[i]) : tab[i + 1]; }
  __device__ __forceinline__ float u(int j) const {
    return stream ? expf(tab[rows - 1] - tab[j]) : tab[rows - 1 - j];
  }
  __device__ __forceinline__ float closing() const { return stream ? expf(tab[rows - 1]) : tab[rows]; }
};

// Fill `tab` for retention r of head h and the tile at token t0 (rows valid
// rows), visible after the next barrier.
__device__ TileWeights fill_weights(float* tab, const ScanF32Params& p, int r, int bh, int t0, int rows) {
  const int h = bh % p.H;
  TileWeights tw{tab, p.las[r] != nullptr, rows};
  if (tw.stream) {
    if (threadIdx.x == 0) {
      const float* s = p.las[r] + static_cast<size_t>(bh) * p.T + t0;
      float run = 0.f;
      for (int i = 0; i < p.TL; ++i) {
        if (i < rows) run += __ldg(s + i);
        tab[i] = run;
      }
      tab[p.TL] = run;
    }
  } else {
    const float* la = p.la[r];
    const float a = la ? __ldg(la + h) : 0.f;
    for (int x = threadIdx.x; x <= p.TL; x += blockDim.x) tab[x] = la ? expf(a * static_cast<float>(x)) : 1.f;
  }
  return tw;
}

// dst[f][c] = sum_{j < rows} wt(j) a[j][f] b[j][c], wt(j) = u(j) (key
// weights) or c(j) (carries); dst is a contiguous [Dk][Dv] state.
__device__ void weighted_outer(float* dst, const float* a, int lda, const float* b, int ldb, const TileWeights& tw,
                               int rows, bool key_weights, int Dk, int Dv) {
  for (int e = threadIdx.x; e < Dk * Dv; e += blockDim.x) {
    const int f = e / Dv, c = e - (e / Dv) * Dv;
    float acc = 0.f;
    for (int j = 0; j < rows; ++j) {
      const float w = key_weights ? tw.u(j) : tw.c(j);
      acc = fmaf(w * a[j * lda + f], b[j * ldb + c], acc);
    }
    dst[e] = acc;
  }
}

__device__ __forceinline__ size_t f32_tile_index(const ScanF32Params& p, int bh, int n, int r) {
  return (static_cast<size_t>(bh) * p.NT + n) * p.R + r;
}

// sc[i][j] = q_i . k_j on the causal triangle of the tile, zero elsewhere.
__device__ void tile_scores(float* sc, const float* sq, const float* sk, int ldk, int Dk, int rows, int TL) {
  for (int e = threadIdx.x; e < TL * TL; e += blockDim.x) {
    const int i = e / TL, j = e - (e / TL) * TL;
    float s = 0.f;
    if (j <= i && i < rows)
      for (int f = 0; f < Dk; ++f) s = fmaf(sq[i * ldk + f], sk[j * ldk + f], s);
    sc[e] = s;
  }
}

// Stage a contiguous [Dk][Dv] state into shared memory with leading dimension ld.
__device__ void stage_state(float* st, int ld, const float* src, int Dk, int Dv) {
  for (int e = threadIdx.x; e < Dk * Dv; e += blockDim.x) {
    const int f = e / Dv, c = e - (e / Dv) * Dv;
    st[f * ld + c] = src[e];
  }
}

}  // namespace

// Forward (1): the local update of tile n (n < NT-1; the last tile's is unused).
__global__ void __launch_bounds__(kF32Threads) scan_f32_state_kernel(ScanF32Params p) {
  extern __shared__ __align__(16) float f32sm[];
  const int n = blockIdx.x, bh = blockIdx.y, b = bh / p.H, h = bh % p.H;
  const int TL = p.TL, Dk = p.Dk, Dv = p.Dv, ldk = odd_ld(Dk), ldv = odd_ld(Dv);
  const int t0 = n * TL, rows = min(TL, p.T - t0);
  (void)h;
  float* sk = f32sm;
  float* sv = sk + TL * ldk;
  float* ex = sv + TL * ldv;
  load_tile_f32(sk, ldk, p.k + b * p.ks[0] + h * p.ks[1] + t0 * p.ks[2], p.ks[2], rows, TL, Dk, Dk, 0.f);
  load_tile_f32(sv, ldv, p.v + b * p.vs[0] + h * p.vs[1] + t0 * p.vs[2], p.vs[2], rows, TL, Dv - p.v_unit, Dv, 1.f);
  for (int r = 0; r < p.R; ++r) {
    __syncthreads();
    const TileWeights tw = fill_weights(ex, p, r, bh, t0, rows);
    __syncthreads();
    if (tw.stream && threadIdx.x == 0) p.closing[f32_tile_index(p, bh, n, r)] = tw.closing();
    weighted_outer(p.states + f32_state_offset(p, bh, n, r), sk, ldk, sv, ldv, tw, rows, true, Dk, Dv);
  }
}

// Forward (2): in place, states[n] <- the state entering tile n, for one
// state element per thread.  Every tile but the last is full, so its closing
// factor is exp(la TL).
__global__ void __launch_bounds__(kF32Threads) scan_f32_prefix_kernel(ScanF32Params p) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  const int bh = blockIdx.y / p.R, r = blockIdx.y % p.R, h = bh % p.H;
  if (e >= p.Dk * p.Dv) return;
  const bool stream = p.las[r] != nullptr;
  const float C = p.la[r] ? expf(__ldg(p.la[r] + h) * static_cast<float>(p.TL)) : 1.f;
  float run = 0.f;
  for (int n = 0; n < p.NT; ++n) {
    float* s = p.states + f32_state_offset(p, bh, n, r) + e;
    const float local = n + 1 < p.NT ? *s : 0.f;
    *s = run;
    const float Cn = stream ? (n + 1 < p.NT ? p.closing[f32_tile_index(p, bh, n, r)] : 0.f) : C;
    run = fmaf(Cn, run, local);
  }
}

// Forward (3): the outputs of tile n for every retention.
__global__ void __launch_bounds__(kF32Threads) scan_f32_out_kernel(ScanF32Params p) {
  extern __shared__ __align__(16) float f32sm[];
  const int n = blockIdx.x, bh = blockIdx.y, b = bh / p.H, h = bh % p.H;
  const int TL = p.TL, Dk = p.Dk, Dv = p.Dv, ldk = odd_ld(Dk), ldv = odd_ld(Dv);
  const int t0 = n * TL, rows = min(TL, p.T - t0);
  float* sq = f32sm;
  float* sk = sq + TL * ldk;
  float* sv = sk + TL * ldk;
  float* sc = sv + TL * ldv;
  float* st = sc + TL * TL;
  float* ex = st + Dk * ldv;
  load_tile_f32(sq, ldk, p.q + b * p.qs[0] + h * p.qs[1] + t0 * p.qs[2], p.qs[2], rows, TL, Dk, Dk, 0.f);
  load_tile_f32(sk, ldk, p.k + b * p.ks[0] + h * p.ks[1] + t0 * p.ks[2], p.ks[2], rows, TL, Dk, Dk, 0.f);
  load_tile_f32(sv, ldv, p.v + b * p.vs[0] + h * p.vs[1] + t0 * p.vs[2], p.vs[2], rows, TL, Dv - p.v_unit, Dv, 1.f);
  __syncthreads();
  tile_scores(sc, sq, sk, ldk, Dk, rows, TL);
  for (int r = 0; r < p.R; ++r) {
    __syncthreads();
    const TileWeights tw = fill_weights(ex, p, r, bh, t0, rows);
    stage_state(st, ldv, p.states + f32_state_offset(p, bh, n, r), Dk, Dv);
    __syncthreads();
    float* out = p.out[r] + (static_cast<size_t>(bh) * p.T + t0) * Dv;
    for (int e = threadIdx.x; e < rows * Dv; e += blockDim.x) {
      const int i = e / Dv, c = e - (e / Dv) * Dv;
      float intra = 0.f;
      for (int j = 0; j <= i; ++j) intra = fmaf(tw.w(i, j) * sc[i * TL + j], sv[j * ldv + c], intra);
      float carry = 0.f;
      for (int f = 0; f < Dk; ++f) carry = fmaf(sq[i * ldk + f], st[f * ldv + c], carry);
      out[e] = fmaf(tw.c(i), carry, intra);
    }
  }
}

// Backward (1): the local read gradient sum_i c(i) q_i^T dout_i of tile n
// (n >= 1; the first tile's only feeds the gradient of the zero initial state).
__global__ void __launch_bounds__(kF32Threads) scan_f32_bwd_state_kernel(ScanF32Params p) {
  extern __shared__ __align__(16) float f32sm[];
  const int n = blockIdx.x + 1, bh = blockIdx.y, b = bh / p.H, h = bh % p.H;
  const int TL = p.TL, Dk = p.Dk, Dv = p.Dv, ldk = odd_ld(Dk), ldv = odd_ld(Dv);
  const int t0 = n * TL, rows = min(TL, p.T - t0);
  (void)h;
  float* sq = f32sm;
  float* sd = sq + TL * ldk;
  float* ex = sd + TL * ldv;
  load_tile_f32(sq, ldk, p.q + b * p.qs[0] + h * p.qs[1] + t0 * p.qs[2], p.qs[2], rows, TL, Dk, Dk, 0.f);
  for (int r = 0; r < p.R; ++r) {
    __syncthreads();
    const TileWeights tw = fill_weights(ex, p, r, bh, t0, rows);
    load_tile_f32(sd, ldv, p.dout[r] + (static_cast<size_t>(bh) * p.T + t0) * Dv, Dv, rows, TL, Dv, Dv, 0.f);
    __syncthreads();
    weighted_outer(p.gstates + f32_state_offset(p, bh, n, r), sq, ldk, sd, ldv, tw, rows, false, Dk, Dv);
  }
}

// Backward (2): in place, gstates[n] <- G(n), the gradient of the state
// leaving tile n, and the closing term sum_n TL C <G(n), S_in(n)> of d la
// (G of the last tile is zero, so only full tiles contribute).
__global__ void __launch_bounds__(kF32Threads) scan_f32_bwd_prefix_kernel(ScanF32Params p) {
  __shared__ float red[32];
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  const int bh = blockIdx.y / p.R, r = blockIdx.y % p.R, h = bh % p.H;
  const bool active = e < p.Dk * p.Dv;
  const float la = p.la[r] ? __ldg(p.la[r] + h) : 0.f;
  const float C = p.la[r] ? expf(la * static_cast<float>(p.TL)) : 1.f;
  float run = 0.f, closing = 0.f;
  if (p.las[r] != nullptr) {
    // per-token stream: per-tile closings; each tile's closing term
    // C_n <G(n), S_in(n)> (block-summed per tile) for the tile kernel
    const bool want = p.dlas[r] != nullptr;
    for (int n = p.NT - 1; n >= 0; --n) {
      const size_t o = f32_state_offset(p, bh, n, r) + e;
      const float Cn = n + 1 < p.NT ? p.closing[f32_tile_index(p, bh, n, r)] : 0.f;
      float term = 0.f;
      if (active) {
        const float local = n >= 1 ? p.gstates[o] : 0.f;
        p.gstates[o] = run;
        term = Cn * run * p.states[o];
        run = fmaf(Cn, run, local);
      }
      if (want) {
        const float tot = block_sum(term, red);
        if (threadIdx.x == 0 && tot != 0.f) atomicAdd(p.zterm + f32_tile_index(p, bh, n, r), tot);
      }
    }
    return;
  }
  if (active) {
    for (int n = p.NT - 1; n >= 0; --n) {
      const size_t o = f32_state_offset(p, bh, n, r) + e;
      const float local = n >= 1 ? p.gstates[o] : 0.f;
      p.gstates[o] = run;
      closing = fmaf(run, p.states[o], closing);
      run = fmaf(C, run, local);
    }
  }
  if (p.la[r] && p.dla[r]) {
    const float tot = block_sum(closing, red);
    if (threadIdx.x == 0) atomicAdd(p.dla[r] + h, static_cast<float>(p.TL) * C * tot);
  }
}

// Backward (3): dq, dk, dv of tile n and its intra, carry and key-weight
// terms of d la.  Each thread owns the same gradient elements in every pass
// (element e of the tile's rows), so the passes accumulate into the outputs
// without synchronisation.
__global__ void __launch_bounds__(kF32Threads) scan_f32_bwd_tile_kernel(ScanF32Params p) {
  extern __shared__ __align__(16) float f32sm[];
  __shared__ float red[32];
  const int n = blockIdx.x, bh = blockIdx.y, b = bh / p.H, h = bh % p.H;
  const int TL = p.TL, Dk = p.Dk, Dv = p.Dv, ldk = odd_ld(Dk), ldv = odd_ld(Dv);
  const int t0 = n * TL, rows = min(TL, p.T - t0);
  float* sq = f32sm;
  float* sk = sq + TL * ldk;
  float* sv = sk + TL * ldk;
  float* sd = sv + TL * ldv;
  float* sc = sd + TL * ldv;
  float* ds = sc + TL * TL;
  float* st = ds + TL * TL;
  float* ex = st + Dk * ldv;
  float* dl = ex + TL + 1;   // per-row log-phase gradient of a stream retention
  const size_t row0 = static_cast<size_t>(bh) * p.T + t0;
  float* dq = p.dq + row0 * Dk;
  float* dk = p.dk + row0 * Dk;
  float* dv = p.dv + row0 * Dv;
  load_tile_f32(sq, ldk, p.q + b * p.qs[0] + h * p.qs[1] + t0 * p.qs[2], p.qs[2], rows, TL, Dk, Dk, 0.f);
  load_tile_f32(sk, ldk, p.k + b * p.ks[0] + h * p.ks[1] + t0 * p.ks[2], p.ks[2], rows, TL, Dk, Dk, 0.f);
  load_tile_f32(sv, ldv, p.v + b * p.vs[0] + h * p.vs[1] + t0 * p.vs[2], p.vs[2], rows, TL, Dv - p.v_unit, Dv, 1.f);
  for (int e = threadIdx.x; e < TL * TL; e += blockDim.x) ds[e] = 0.f;
  for (int e = threadIdx.x; e < rows * Dk; e += blockDim.x) dq[e] = dk[e] = 0.f;
  for (int e = threadIdx.x; e < rows * Dv; e += blockDim.x) dv[e] = 0.f;
  __syncthreads();
  tile_scores(sc, sq, sk, ldk, Dk, rows, TL);
  for (int r = 0; r < p.R; ++r) {
    const bool stream = p.las[r] != nullptr;
    const bool want = !stream && p.la[r] != nullptr && p.dla[r] != nullptr;
    const bool want_s = stream && p.dlas[r] != nullptr;
    __syncthreads();
    const TileWeights tw = fill_weights(ex, p, r, bh, t0, rows);
    load_tile_f32(sd, ldv, p.dout[r] + row0 * Dv, Dv, rows, TL, Dv, Dv, 0.f);
    stage_state(st, ldv, p.states + f32_state_offset(p, bh, n, r), Dk, Dv);
    if (want_s)
      for (int i = threadIdx.x; i < TL; i += blockDim.x) dl[i] = 0.f;
    __syncthreads();
    float dla = 0.f;
    // g = dout v^T on the causal triangle: ds += w o g, intra term of d la
    for (int e = threadIdx.x; e < TL * TL; e += blockDim.x) {
      const int i = e / TL, j = e - (e / TL) * TL;
      if (j <= i && i < rows) {
        float g = 0.f;
        for (int c = 0; c < Dv; ++c) g = fmaf(sd[i * ldv + c], sv[j * ldv + c], g);
        const float w = tw.w(i, j);
        ds[e] = fmaf(w, g, ds[e]);
        if (want) dla = fmaf(static_cast<float>(i - j) * w * sc[e], g, dla);
        if (want_s && j < i) {
          const float x = w * sc[e] * g;   // d/dl_i of w(i,j) is +w, d/dl_j is -w
          atomicAdd(dl + i, x);
          atomicAdd(dl + j, -x);
        }
      }
    }
    // dv_j += sum_{i>=j} w (q_i.k_j) dout_i
    for (int e = threadIdx.x; e < rows * Dv; e += blockDim.x) {
      const int j = e / Dv, c = e - (e / Dv) * Dv;
      float acc = 0.f;
      for (int i = j; i < rows; ++i) acc = fmaf(tw.w(i, j) * sc[i * TL + j], sd[i * ldv + c], acc);
      dv[e] += acc;
    }
    // a_i = S_in dout_i: dq_i += c(i) a_i, carry term of d la
    for (int e = threadIdx.x; e < rows * Dk; e += blockDim.x) {
      const int i = e / Dk, f = e - (e / Dk) * Dk;
      float a = 0.f;
      for (int c = 0; c < Dv; ++c) a = fmaf(st[f * ldv + c], sd[i * ldv + c], a);
      const float cc = tw.c(i);
      dq[e] = fmaf(cc, a, dq[e]);
      if (want) dla = fmaf(static_cast<float>(i + 1) * cc * sq[i * ldk + f], a, dla);
      if (want_s) atomicAdd(dl + i, cc * sq[i * ldk + f] * a);
    }
    __syncthreads();
    stage_state(st, ldv, p.gstates + f32_state_offset(p, bh, n, r), Dk, Dv);
    __syncthreads();
    // b_j = G v_j: dk_j += u(j) b_j, key-weight term of d la
    for (int e = threadIdx.x; e < rows * Dk; e += blockDim.x) {
      const int j = e / Dk, f = e - (e / Dk) * Dk;
      float bj = 0.f;
      for (int c = 0; c < Dv; ++c) bj = fmaf(st[f * ldv + c], sv[j * ldv + c], bj);
      const float u = tw.u(j);
      dk[e] = fmaf(u, bj, dk[e]);
      if (want) dla = fmaf(static_cast<float>(rows - 1 - j) * u * sk[j * ldk + f], bj, dla);
      if (want_s && j < rows - 1) {
        // d/dl_last of u(j) is +u(j), d/dl_j is -u(j)
        const float x = u * sk[j * ldk + f] * bj;
        atomicAdd(dl + rows - 1, x);
        atomicAdd(dl + j, -x);
      }
    }
    // dv_j += u(j) k_j G
    for (int e = threadIdx.x; e < rows * Dv; e += blockDim.x) {
      const int j = e / Dv, c = e - (e / Dv) * Dv;
      float kg = 0.f;
      for (int f = 0; f < Dk; ++f) kg = fmaf(sk[j * ldk + f], st[f * ldv + c], kg);
      dv[e] = fmaf(tw.u(j), kg, dv[e]);
    }
    if (want) {
      const float tot = block_sum(dla, red);
      if (threadIdx.x == 0) atomicAdd(p.dla[r] + h, tot);
    }
    if (want_s) {
      // the tile's closing term on its last row, then d la_t = sum_{i>=t} dl_i
      __syncthreads();
      if (threadIdx.x == 0) {
        float run = p.zterm[f32_tile_index(p, bh, n, r)];
        float* out = p.dlas[r] + row0;
        for (int t = rows - 1; t >= 0; --t) {
          run += dl[t];
          out[t] = run;
        }
      }
    }
  }
  __syncthreads();
  // dq_i += sum_{j<=i} ds_ij k_j;  dk_j += sum_{i>=j} ds_ij q_i
  for (int e = threadIdx.x; e < rows * Dk; e += blockDim.x) {
    const int i = e / Dk, f = e - (e / Dk) * Dk;
    float aq = 0.f, ak = 0.f;
    for (int j = 0; j <= i; ++j) aq = fmaf(ds[i * TL + j], sk[j * ldk + f], aq);
    for (int t = i; t < rows; ++t) ak = fmaf(ds[t * TL + i], sq[t * ldk + f], ak);
    dq[e] += aq;
    dk[e] += ak;
  }
}

size_t scan_f32_smem(int TL, int Dk, int Dv, bool backward) {
  const size_t ldk = odd_ld(Dk), ldv = odd_ld(Dv);
  const size_t tiles = 2 * TL * ldk + (backward ? 2 : 1) * TL * ldv;
  const size_t scores = (backward ? 2 : 1) * static_cast<size_t>(TL) * TL;
  return (tiles + scores + Dk * ldv + TL + 1 + (backward ? TL : 0)) * sizeof(float);
}

static size_t state_kernel_smem(const ScanF32Params& p) {
  return (static_cast<size_t>(p.TL) * (odd_ld(p.Dk) + odd_ld(p.Dv)) + p.TL + 1) * sizeof(float);
}

static int set_smem(const void* fn, size_t bytes) {
  const cudaError_t e =
      cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
  if (e != cudaSuccess)
    return set_error(TS_ERR_CUDA, "scan_f32: shared memory of %zu bytes: %s", bytes, cudaGetErrorString(e));
  return TS_OK;
}

int launch_scan_f32_fwd(const ScanF32Params& p, cudaStream_t s) {
  const int BH = p.B * p.H;
  const size_t sm_state = state_kernel_smem(p), sm_out = scan_f32_smem(p.TL, p.Dk, p.Dv, false);
  if (int e = set_smem(reinterpret_cast<const void*>(scan_f32_state_kernel), sm_state)) return e;
  if (int e = set_smem(reinterpret_cast<const void*>(scan_f32_out_kernel), sm_out)) return e;
  if (p.NT > 1) {
    scan_f32_state_kernel<<<dim3(p.NT - 1, BH), kF32Threads, sm_state, s>>>(p);
    if (int e = check_launch("scan_f32_state_kernel")) return e;
  }
  scan_f32_prefix_kernel<<<dim3(ceil_div(p.Dk * p.Dv, kF32Threads), BH * p.R), kF32Threads, 0, s>>>(p);
  if (int e = check_launch("scan_f32_prefix_kernel")) return e;
  scan_f32_out_kernel<<<dim3(p.NT, BH), kF32Threads, sm_out, s>>>(p);
  return check_launch("scan_f32_out_kernel");
}

int launch_scan_f32_bwd(const ScanF32Params& p, cudaStream_t s) {
  const int BH = p.B * p.H;
  const size_t sm_state = state_kernel_smem(p), sm_tile = scan_f32_smem(p.TL, p.Dk, p.Dv, true);
  if (int e = set_smem(reinterpret_cast<const void*>(scan_f32_bwd_state_kernel), sm_state)) return e;
  if (int e = set_smem(reinterpret_cast<const void*>(scan_f32_bwd_tile_kernel), sm_tile)) return e;
  if (p.NT > 1) {
    scan_f32_bwd_state_kernel<<<dim3(p.NT - 1, BH), kF32Threads, sm_state, s>>>(p);
    if (int e = check_launch("scan_f32_bwd_state_kernel")) return e;
  }
  if (p.zterm != nullptr) {
    const cudaError_t e = cudaMemsetAsync(p.zterm, 0, static_cast<size_t>(BH) * p.NT * p.R * sizeof(float), s);
    if (e != cudaSuccess) return set_error(TS_ERR_CUDA, "scan_f32: %s", cudaGetErrorString(e));
  }
  scan_f32_bwd_prefix_kernel<<<dim3(ceil_div(p.Dk * p.Dv, kF32Threads), BH * p.R), kF32Threads, 0, s>>>(p);
  if (int e = check_launch("scan_f32_bwd_prefix_kernel")) return e;
  scan_f32_bwd_tile_kernel<<<dim3(p.NT, BH), kF32Threads, sm_tile, s>>>(p);
  return check_launch("scan_f32_bwd_tile_kernel");
}

}  // namespace ts
