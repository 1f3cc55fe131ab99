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

// ex[x] = exp(la_h x) for x in [0, TL]; all ones for the plain sum.
__device__ void fill_exp(float* ex, const float* la, int h, int TL) {
  const float a = la ? __ldg(la + h) : 0.f;
  for (int x = threadIdx.x; x <= TL; x += blockDim.x) ex[x] = la ? expf(a * static_cast<float>(x)) : 1.f;
}

// dst[f][c] = sum_{j < rows} wt(j) a[j][f] b[j][c], wt(j) = ex[rows-1-j]
// (key weights) or ex[j+1] (carries); dst is a contiguous [Dk][Dv] state.
__device__ void weighted_outer(float* dst, const float* a, int lda, const float* b, int ldb, const float* ex,
                               int rows, bool key_weights, int Dk, int Dv) {
  for (int e = threadIdx.x; e < Dk * Dv; e += blockDim.x) {
    const int f = e / Dv, c = e - (e / Dv) * Dv;
    float acc = 0.f;
    for (int j = 0; j < rows; ++j) {
      const float w = ex[key_weights ? rows - 1 - j : j + 1];
      acc = fmaf(w * a[j * lda + f], b[j * ldb + c], acc);
    }
    dst[e] = acc;
  }
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
  float* sk = f32sm;
  float* sv = sk + TL * ldk;
  float* ex = sv + TL * ldv;
  load_tile_f32(sk, ldk, p.k + b * p.ks[0] + h * p.ks[1] + t0 * p.ks[2], p.ks[2], rows, TL, Dk, Dk, 0.f);
  load_tile_f32(sv, ldv, p.v + b * p.vs[0] + h * p.vs[1] + t0 * p.vs[2], p.vs[2], rows, TL, Dv - p.v_unit, Dv, 1.f);
  for (int r = 0; r < p.R; ++r) {
    __syncthreads();
    fill_exp(ex, p.la[r], h, TL);
    __syncthreads();
    weighted_outer(p.states + f32_state_offset(p, bh, n, r), sk, ldk, sv, ldv, ex, rows, true, Dk, Dv);
  }
}

// Forward (2): in place, states[n] <- the state entering tile n, for one
// state element per thread.  Every tile but the last is full, so its closing
// factor is exp(la TL).
__global__ void __launch_bounds__(kF32Threads) scan_f32_prefix_kernel(ScanF32Params p) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  const int bh = blockIdx.y / p.R, r = blockIdx.y % p.R, h = bh % p.H;
  if (e >= p.Dk * p.Dv) return;
  const float C = p.la[r] ? expf(__ldg(p.la[r] + h) * static_cast<float>(p.TL)) : 1.f;
  float run = 0.f;
  for (int n = 0; n < p.NT; ++n) {
    float* s = p.states + f32_state_offset(p, bh, n, r) + e;
    const float local = n + 1 < p.NT ? *s : 0.f;
    *s = run;
    run = fmaf(C, run, local);
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
    fill_exp(ex, p.la[r], h, TL);
    stage_state(st, ldv, p.states + f32_state_offset(p, bh, n, r), Dk, Dv);
    __syncthreads();
    float* out = p.out[r] + (static_cast<size_t>(bh) * p.T + t0) * Dv;
    for (int e = threadIdx.x; e < rows * Dv; e += blockDim.x) {
      const int i = e / Dv, c = e - (e / Dv) * Dv;
      float intra = 0.f;
      for (int j = 0; j <= i; ++j) intra = fmaf(ex[i - j] * sc[i * TL + j], sv[j * ldv + c], intra);
      float carry = 0.f;
      for (int f = 0; f < Dk; ++f) carry = fmaf(sq[i * ldk + f], st[f * ldv + c], carry);
      out[e] = fmaf(ex[i + 1], carry, intra);
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
  float* sq = f32sm;
  float* sd = sq + TL * ldk;
  float* ex = sd + TL * ldv;
  load_tile_f32(sq, ldk, p.q + b * p.qs[0] + h * p.qs[1] + t0 * p.qs[2], p.qs[2], rows, TL, Dk, Dk, 0.f);
  for (int r = 0; r < p.R; ++r) {
    __syncthreads();
    fill_exp(ex, p.la[r], h, TL);
    load_tile_f32(sd, ldv, p.dout[r] + (static_cast<size_t>(bh) * p.T + t0) * Dv, Dv, rows, TL, Dv, Dv, 0.f);
    __syncthreads();
    weighted_outer(p.gstates + f32_state_offset(p, bh, n, r), sq, ldk, sd, ldv, ex, rows, false, Dk, Dv);
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
    const bool want = p.la[r] != nullptr && p.dla[r] != nullptr;
    __syncthreads();
    fill_exp(ex, p.la[r], h, TL);
    load_tile_f32(sd, ldv, p.dout[r] + row0 * Dv, Dv, rows, TL, Dv, Dv, 0.f);
    stage_state(st, ldv, p.states + f32_state_offset(p, bh, n, r), Dk, Dv);
    __syncthreads();
    float dla = 0.f;
    // g = dout v^T on the causal triangle: ds += w o g, intra term of d la
    for (int e = threadIdx.x; e < TL * TL; e += blockDim.x) {
      const int i = e / TL, j = e - (e / TL) * TL;
      if (j <= i && i < rows) {
        float g = 0.f;
        for (int c = 0; c < Dv; ++c) g = fmaf(sd[i * ldv + c], sv[j * ldv + c], g);
        const float w = ex[i - j];
        ds[e] = fmaf(w, g, ds[e]);
        if (want) dla = fmaf(static_cast<float>(i - j) * w * sc[e], g, dla);
      }
    }
    // dv_j += sum_{i>=j} w (q_i.k_j) dout_i
    for (int e = threadIdx.x; e < rows * Dv; e += blockDim.x) {
      const int j = e / Dv, c = e - (e / Dv) * Dv;
      float acc = 0.f;
      for (int i = j; i < rows; ++i) acc = fmaf(ex[i - j] * sc[i * TL + j], sd[i * ldv + c], acc);
      dv[e] += acc;
    }
    // a_i = S_in dout_i: dq_i += c(i) a_i, carry term of d la
    for (int e = threadIdx.x; e < rows * Dk; e += blockDim.x) {
      const int i = e / Dk, f = e - (e / Dk) * Dk;
      float a = 0.f;
      for (int c = 0; c < Dv; ++c) a = fmaf(st[f * ldv + c], sd[i * ldv + c], a);
      const float cc = ex[i + 1];
      dq[e] = fmaf(cc, a, dq[e]);
      if (want) dla = fmaf(static_cast<float>(i + 1) * cc * sq[i * ldk + f], a, dla);
    }
    __syncthreads();
    stage_state(st, ldv, p.gstates + f32_state_offset(p, bh, n, r), Dk, Dv);
    __syncthreads();
    // b_j = G v_j: dk_j += u(j) b_j, key-weight term of d la
    for (int e = threadIdx.x; e < rows * Dk; e += blockDim.x) {
      const int j = e / Dk, f = e - (e / Dk) * Dk;
      float bj = 0.f;
      for (int c = 0; c < Dv; ++c) bj = fmaf(st[f * ldv + c], sv[j * ldv + c], bj);
      const float u = ex[rows - 1 - j];
      dk[e] = fmaf(u, bj, dk[e]);
      if (want) dla = fmaf(static_cast<float>(rows - 1 - j) * u * sk[j * ldk + f], bj, dla);
    }
    // dv_j += u(j) k_j G
    for (int e = threadIdx.x; e < rows * Dv; e += blockDim.x) {
      const int j = e / Dv, c = e - (e / Dv) * Dv;
      float kg = 0.f;
      for (int f = 0; f < Dk; ++f) kg = fmaf(sk[j * ldk + f], st[f * ldv + c], kg);
      dv[e] = fmaf(ex[rows - 1 - j], kg, dv[e]);
    }
    if (want) {
      const float tot = block_sum(dla, red);
      if (threadIdx.x == 0) atomicAdd(p.dla[r] + h, tot);
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
  return (tiles + scores + Dk * ldv + TL + 1) * sizeof(float);
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
  scan_f32_bwd_prefix_kernel<<<dim3(ceil_div(p.Dk * p.Dv, kF32Threads), BH * p.R), kF32Threads, 0, s>>>(p);
  if (int e = check_launch("scan_f32_bwd_prefix_kernel")) return e;
  scan_f32_bwd_tile_kernel<<<dim3(p.NT, BH), kF32Threads, sm_tile, s>>>(p);
  return check_launch("scan_f32_bwd_tile_kernel");
}

}  // namespace ts
