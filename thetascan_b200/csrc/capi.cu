// C-ABI entry points: argument validation, workspace sizing and launches.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "capi_internal.h"
#include "scan.cuh"
#include "scan_f32.cuh"

namespace ts {

namespace {
thread_local int g_last_code = TS_OK;
thread_local char g_last_msg[512] = "";
constexpr size_t kMaxSmem = 232448;  // 227 KB opt-in per block on sm_100
}  // namespace

int set_error(int code, const char* fmt, ...) {
  g_last_code = code;
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_msg, sizeof(g_last_msg), fmt, ap);
  va_end(ap);
  return code;
}

namespace {
std::atomic<long long> g_launches{0};
}  // namespace

int check_launch(const char* what) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(TS_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return TS_OK;
}

int launch_scan_fwd(const ScanParams& p, cudaStream_t s, bool tile_states, bool outputs);
int launch_scan_bwd(const ScanParams& p, const ScanGradParams& g, cudaStream_t s, bool tile_terms, bool grads);
size_t scan_state_smem(const ScanParams& p);
size_t scan_out_smem(const ScanParams& p);
size_t scan_bwd_max_smem(const ScanParams& p);

static size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

static size_t states_bytes(const ScanParams& p) {
  return align256(static_cast<size_t>(p.B) * p.H * p.NT * p.R * p.DkM * p.DvP * sizeof(float));
}
static size_t images_bytes(const ScanParams& p) {
  return align256(static_cast<size_t>(p.B) * p.H * p.NT * p.R * p.DvP * p.DkP * 2);
}
// Segment totals of the backward's two-level tile prefix (zero when unused).
static size_t segs_bytes(const ScanParams& p) {
  return align256(static_cast<size_t>(p.B) * p.H * p.R * p.NS * p.DkM * p.DvP * sizeof(float));
}

// Validate `a` and fill `p` (workspace pointers left null).
static int build_scan_params(const ts_scan_args* a, ScanParams* p) {
  if (!a) return set_error(TS_ERR_VALUE, "scan: null arguments");
  if (a->batch < 1 || a->heads < 1 || a->tokens < 1)
    return set_error(TS_ERR_VALUE, "scan: batch, heads and tokens must be >= 1");
  if (a->dk < 1 || a->dk > 256)
    return set_error(TS_ERR_NOT_IMPLEMENTED, "scan: key width %d outside 1..256", a->dk);
  if (a->v_append_unit < 0 || a->v_append_unit > 2)
    return set_error(TS_ERR_VALUE, "scan: v_append_unit must be 0, 1 or 2");
  if (a->dv < 1 + a->v_append_unit || a->dv > 256)
    return set_error(TS_ERR_NOT_IMPLEMENTED, "scan: payload width %d outside 1..256", a->dv);
  if (a->n_retentions < 1 || a->n_retentions > TS_MAX_RETENTIONS)
    return set_error(TS_ERR_VALUE, "scan: n_retentions must be in 1..%d", TS_MAX_RETENTIONS);
  if (!a->q || !a->k || !a->v) return set_error(TS_ERR_VALUE, "scan: null stream pointer");
  for (int r = 0; r < TS_MAX_RETENTIONS && r < a->n_retentions; ++r)
    if (a->log_alpha_stream[r])
      return set_error(TS_ERR_NOT_IMPLEMENTED,
                       "scan: per-token retention streams take f32 streams (f32_streams), on the CUDA cores");
  if (a->out_dtype != TS_DTYPE_F32 && a->out_dtype != TS_DTYPE_BF16)
    return set_error(TS_ERR_VALUE, "scan: out_dtype must be TS_DTYPE_F32 or TS_DTYPE_BF16");
  std::memset(p, 0, sizeof(*p));
  p->B = a->batch;
  p->H = a->heads;
  p->T = a->tokens;
  p->Dk = a->dk;
  p->Dv = a->dv;
  p->DkP = round_up(a->dk, 16);
  p->DkM = round_up(a->dk, 128);
  p->DvP = round_up(a->dv, 16);
  p->NT = ceil_div(a->tokens, 128);
  p->RU = a->n_retentions;
  p->q = static_cast<const __nv_bfloat16*>(a->q);
  p->k = static_cast<const __nv_bfloat16*>(a->k);
  p->v = static_cast<const __nv_bfloat16*>(a->v);
  for (int i = 0; i < 3; ++i) {
    p->qs[i] = a->q_strides[i];
    p->ks[i] = a->k_strides[i];
    p->vs[i] = a->v_strides[i];
  }
  p->v_unit = a->v_append_unit;
  // Caller slots first, then one auxiliary decayed slot per stale slot.
  p->R = p->RU;
  for (int r = 0; r < p->RU; ++r) {
    p->la[r] = a->log_alpha[r];
    p->out[r] = a->out[r];
    p->kind[r] = kSlotDecay;
    p->partner[r] = -1;
    if (!a->out[r]) return set_error(TS_ERR_VALUE, "scan: null output pointer for retention %d", r);
    if (a->stale[r]) {
      if (!a->log_alpha[r]) return set_error(TS_ERR_VALUE, "scan: stale retention %d needs a log_alpha", r);
      const int aux = p->R++;
      p->kind[r] = kSlotStale;
      p->partner[r] = aux;
      p->la[aux] = a->log_alpha[r];
      p->kind[aux] = kSlotAux;
      p->partner[aux] = r;
      p->out[aux] = nullptr;
      p->any_stale = 1;
    }
  }
  p->out_bf16 = a->out_dtype == TS_DTYPE_BF16;
  if (a->stage < 0 || a->stage > 2) return set_error(TS_ERR_VALUE, "scan: stage must be 0, 1 or 2");
  p->NS = prefix_segments(p->NT, p->any_stale != 0);
  if (p->any_stale && (a->init_state || a->final_state || a->stage != 0))
    return set_error(TS_ERR_NOT_IMPLEMENTED, "scan: stale retentions take no boundary states or stages");
  p->init = a->init_state;
  p->final_state = a->final_state;
  p->all_tiles = a->final_state != nullptr;
  p->store = 1;
  const int mblocks = p->DkM / 128;
  // TMEM columns: score plus every caller slot's read (output kernel), the
  // tile update and its la-weighted copy (state kernels), score, g and dv
  // (dv kernel).
  if (128 + p->RU * p->DvP > 512 || 2 * mblocks * p->DvP > 512 || 256 + p->DvP > 512)
    return set_error(TS_ERR_NOT_IMPLEMENTED,
                     "scan: %d retentions of a %dx%d state exceed the 512 tensor-memory columns of one CTA",
                     p->R, p->Dk, p->Dv);
  if (scan_state_smem(*p) > kMaxSmem || scan_out_smem(*p) > kMaxSmem || scan_bwd_max_smem(*p) > kMaxSmem)
    return set_error(TS_ERR_NOT_IMPLEMENTED,
                     "scan: key width %d with payload width %d exceeds the shared-memory budget of one CTA",
                     p->Dk, p->Dv);
  return TS_OK;
}

// ------------------------------------------------------------ f32 streams

static size_t f32_states_bytes(const ScanF32Params& p) {
  return align256(static_cast<size_t>(p.B) * p.H * p.NT * p.R * p.Dk * p.Dv * sizeof(float));
}
// Per-tile scalars of per-token retention streams (closings in the forward
// workspace, closing terms in the backward's), after the states.
static size_t f32_tile_bytes(const ScanF32Params& p) {
  return align256(static_cast<size_t>(p.B) * p.H * p.NT * p.R * sizeof(float));
}

// Validate `a` (f32_streams set) and fill `p` (workspace pointers left null).
static int build_scan_f32_params(const ts_scan_args* a, ScanF32Params* p) {
  if (a->batch < 1 || a->heads < 1 || a->tokens < 1)
    return set_error(TS_ERR_VALUE, "scan: batch, heads and tokens must be >= 1");
  if (a->dk < 1 || a->dk > kF32MaxDk)
    return set_error(TS_ERR_NOT_IMPLEMENTED, "scan (f32 streams): key width %d outside 1..%d", a->dk, kF32MaxDk);
  if (a->v_append_unit < 0 || a->v_append_unit > 2)
    return set_error(TS_ERR_VALUE, "scan: v_append_unit must be 0, 1 or 2");
  if (a->dv < 1 + a->v_append_unit || a->dv > kF32MaxDv)
    return set_error(TS_ERR_NOT_IMPLEMENTED, "scan (f32 streams): payload width %d outside 1..%d", a->dv,
                     kF32MaxDv);
  if (a->n_retentions < 1 || a->n_retentions > TS_MAX_RETENTIONS)
    return set_error(TS_ERR_VALUE, "scan: n_retentions must be in 1..%d", TS_MAX_RETENTIONS);
  if (!a->q || !a->k || !a->v) return set_error(TS_ERR_VALUE, "scan: null stream pointer");
  if (a->out_dtype != TS_DTYPE_F32)
    return set_error(TS_ERR_VALUE, "scan: f32 streams give f32 outputs (out_dtype TS_DTYPE_F32)");
  if (a->init_state || a->final_state || a->stage != 0)
    return set_error(TS_ERR_NOT_IMPLEMENTED, "scan: f32 streams take no boundary states or stages");
  std::memset(p, 0, sizeof(*p));
  p->B = a->batch;
  p->H = a->heads;
  p->T = a->tokens;
  p->Dk = a->dk;
  p->Dv = a->dv;
  // 64-token tiles where the backward's tiles and one staged state fit, else 32
  p->TL = scan_f32_smem(64, a->dk, a->dv, true) <= kMaxSmem ? 64 : 32;
  if (scan_f32_smem(p->TL, a->dk, a->dv, true) > kMaxSmem)
    return set_error(TS_ERR_NOT_IMPLEMENTED,
                     "scan (f32 streams): key width %d with payload width %d exceeds the shared-memory budget of one CTA",
                     a->dk, a->dv);
  p->NT = ceil_div(a->tokens, p->TL);
  p->R = a->n_retentions;
  p->v_unit = a->v_append_unit;
  if (static_cast<long long>(p->B) * p->H * p->R > 65535)
    return set_error(TS_ERR_NOT_IMPLEMENTED, "scan (f32 streams): batch x heads x retentions above 65535");
  p->q = static_cast<const float*>(a->q);
  p->k = static_cast<const float*>(a->k);
  p->v = static_cast<const float*>(a->v);
  for (int i = 0; i < 3; ++i) {
    p->qs[i] = a->q_strides[i];
    p->ks[i] = a->k_strides[i];
    p->vs[i] = a->v_strides[i];
  }
  for (int r = 0; r < p->R; ++r) {
    if (a->stale[r])
      return set_error(TS_ERR_NOT_IMPLEMENTED,
                       "scan: stale retentions of f32 streams are formed by the host (plain read minus recency read)");
    if (!a->out[r]) return set_error(TS_ERR_VALUE, "scan: null output pointer for retention %d", r);
    if (a->log_alpha_stream[r] && a->log_alpha[r])
      return set_error(TS_ERR_VALUE, "scan: retention %d has both a static and a per-token log-retention", r);
    p->la[r] = a->log_alpha[r];
    p->las[r] = a->log_alpha_stream[r];
    p->out[r] = static_cast<float*>(a->out[r]);
  }
  return TS_OK;
}

static int scan_f32_fwd(const ts_scan_args* a, cudaStream_t s) {
  ScanF32Params p;
  if (int e = build_scan_f32_params(a, &p)) return e;
  const size_t need = f32_states_bytes(p) + f32_tile_bytes(p);
  if (!a->workspace || a->workspace_bytes < need)
    return set_error(TS_ERR_VALUE, "scan_fwd: workspace of %zu bytes needed", need);
  p.states = static_cast<float*>(a->workspace);
  p.closing = reinterpret_cast<float*>(static_cast<uint8_t*>(a->workspace) + f32_states_bytes(p));
  return launch_scan_f32_fwd(p, s);
}

static int scan_f32_bwd(const ts_scan_args* a, const ts_scan_grad_args* g, cudaStream_t s) {
  ScanF32Params p;
  if (int e = build_scan_f32_params(a, &p)) return e;
  if (!g) return set_error(TS_ERR_VALUE, "scan_bwd: null gradient arguments");
  const size_t need = f32_states_bytes(p) + f32_tile_bytes(p);
  if (!a->workspace || a->workspace_bytes < need)
    return set_error(TS_ERR_VALUE, "scan_bwd: the forward workspace (%zu bytes) is required", need);
  if (!g->workspace || g->workspace_bytes < need)
    return set_error(TS_ERR_VALUE, "scan_bwd: backward workspace of %zu bytes needed", need);
  if (g->grad_dtype != TS_DTYPE_F32)
    return set_error(TS_ERR_VALUE, "scan_bwd: f32 streams give f32 gradients (grad_dtype TS_DTYPE_F32)");
  if (g->dv_strides[0] | g->dv_strides[1] | g->dv_strides[2])
    return set_error(TS_ERR_NOT_IMPLEMENTED, "scan_bwd: f32 streams write a contiguous dv");
  if (g->dfinal_state || g->dinit_state || g->stage != 0)
    return set_error(TS_ERR_NOT_IMPLEMENTED, "scan_bwd: f32 streams take no boundary states or stages");
  if (!g->dq || !g->dk || !g->dv) return set_error(TS_ERR_VALUE, "scan_bwd: null gradient output");
  bool any_stream = false;
  for (int r = 0; r < p.R; ++r) {
    p.dout[r] = static_cast<const float*>(g->dout[r]);
    if (!p.dout[r]) return set_error(TS_ERR_VALUE, "scan_bwd: null dout for retention %d", r);
    p.dla[r] = g->dlog_alpha[r];
    p.dlas[r] = p.las[r] ? g->dlog_alpha_stream[r] : nullptr;
    any_stream |= p.dlas[r] != nullptr;
  }
  p.dq = static_cast<float*>(g->dq);
  p.dk = static_cast<float*>(g->dk);
  p.dv = static_cast<float*>(g->dv);
  p.states = static_cast<float*>(a->workspace);
  p.closing = reinterpret_cast<float*>(static_cast<uint8_t*>(a->workspace) + f32_states_bytes(p));
  p.gstates = static_cast<float*>(g->workspace);
  p.zterm = any_stream ? reinterpret_cast<float*>(static_cast<uint8_t*>(g->workspace) + f32_states_bytes(p))
                       : nullptr;
  return launch_scan_f32_bwd(p, s);
}

}  // namespace ts

using namespace ts;

extern "C" {

const char* ts_b200_version(void) { return "thetascan_b200 0.1.0 (sm_100a)"; }

long long ts_b200_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int ts_b200_last_error(char* buf, size_t len) {
  if (buf && len) {
    std::strncpy(buf, g_last_msg, len - 1);
    buf[len - 1] = '\0';
  }
  return g_last_code;
}

int ts_b200_device_status(ts_stream_t stream, int* status) {
  cudaError_t e = cudaStreamSynchronize(reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return set_error(TS_ERR_CUDA, "device_status: %s", cudaGetErrorString(e));
  int value = 0, zero = 0;
  e = cudaMemcpyFromSymbol(&value, g_device_status, sizeof(int));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_device_status, &zero, sizeof(int));
  if (e != cudaSuccess) return set_error(TS_ERR_CUDA, "device_status: %s", cudaGetErrorString(e));
  if (status) *status = value;
  if (value) return set_error(TS_ERR_DEVICE, "a kernel gave up on a bounded wait (code %d)", value);
  return TS_OK;
}

int ts_b200_selftest_mma(const void* A, const void* B, float* D, int N, int K, int a_mn, int b_mn,
                         ts_stream_t stream) {
  return selftest_mma(A, B, D, N, K, a_mn, b_mn, reinterpret_cast<cudaStream_t>(stream));
}

int ts_b200_selftest_tma_mma(const void* A, const void* B, float* D, int N, int K, int a_mn, int b_mn,
                             ts_stream_t stream) {
  return selftest_tma_mma(A, B, D, N, K, a_mn, b_mn, reinterpret_cast<cudaStream_t>(stream));
}

size_t ts_b200_scan_workspace_bytes(const ts_scan_args* args) {
  if (args && args->f32_streams) {
    ScanF32Params p;
    return build_scan_f32_params(args, &p) == TS_OK ? f32_states_bytes(p) + f32_tile_bytes(p) : 0;
  }
  ScanParams p;
  if (build_scan_params(args, &p) != TS_OK) return 0;
  return states_bytes(p) + images_bytes(p);
}

size_t ts_b200_scan_bwd_workspace_bytes(const ts_scan_args* args) {
  if (args && args->f32_streams) {
    ScanF32Params p;
    return build_scan_f32_params(args, &p) == TS_OK ? f32_states_bytes(p) + f32_tile_bytes(p) : 0;
  }
  ScanParams p;
  if (build_scan_params(args, &p) != TS_OK) return 0;
  return 2 * states_bytes(p) + images_bytes(p) + segs_bytes(p);
}

int ts_b200_scan_fwd(const ts_scan_args* args, ts_stream_t stream) {
  if (args && args->f32_streams) return scan_f32_fwd(args, reinterpret_cast<cudaStream_t>(stream));
  ScanParams p;
  if (int e = build_scan_params(args, &p)) return e;
  const size_t need = states_bytes(p) + images_bytes(p);
  if (!args->workspace || args->workspace_bytes < need)
    return set_error(TS_ERR_VALUE, "scan_fwd: workspace of %zu bytes needed", need);
  p.states = static_cast<float*>(args->workspace);
  p.images = reinterpret_cast<__nv_bfloat16*>(static_cast<uint8_t*>(args->workspace) + states_bytes(p));
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (args->stage == 1) {
    // tile states of every tile and the final state from a zero initial state
    if (!p.final_state) return set_error(TS_ERR_VALUE, "scan_fwd: stage 1 needs final_state");
    p.init = nullptr;
    p.store = 0;
    p.all_tiles = 1;
    return launch_scan_fwd(p, s, true, false);
  }
  return launch_scan_fwd(p, s, args->stage == 0, true);
}

int ts_b200_scan_bwd(const ts_scan_args* args, const ts_scan_grad_args* grad, ts_stream_t stream) {
  if (args && args->f32_streams) return scan_f32_bwd(args, grad, reinterpret_cast<cudaStream_t>(stream));
  ScanParams p;
  if (int e = build_scan_params(args, &p)) return e;
  if (!grad) return set_error(TS_ERR_VALUE, "scan_bwd: null gradient arguments");
  const size_t need = states_bytes(p) + images_bytes(p);
  if (!args->workspace || args->workspace_bytes < need)
    return set_error(TS_ERR_VALUE, "scan_bwd: the forward workspace (%zu bytes) is required", need);
  const size_t need_bwd = 2 * states_bytes(p) + images_bytes(p) + segs_bytes(p);
  if (!grad->workspace || grad->workspace_bytes < need_bwd)
    return set_error(TS_ERR_VALUE, "scan_bwd: backward workspace of %zu bytes needed", need_bwd);
  if (grad->stage != 1 && (!grad->dq || !grad->dk || !grad->dv))
    return set_error(TS_ERR_VALUE, "scan_bwd: null gradient output");
  p.states = static_cast<float*>(args->workspace);
  p.images = reinterpret_cast<__nv_bfloat16*>(static_cast<uint8_t*>(args->workspace) + states_bytes(p));
  ScanGradParams g;
  std::memset(&g, 0, sizeof(g));
  for (int r = 0; r < p.RU; ++r) {
    g.dout[r] = static_cast<const __nv_bfloat16*>(grad->dout[r]);
    if (!g.dout[r]) return set_error(TS_ERR_VALUE, "scan_bwd: null dout for retention %d", r);
    g.dla[r] = grad->dlog_alpha[r];
  }
  for (int r = p.RU; r < p.R; ++r) g.dla[r] = g.dla[p.partner[r]];
  if (p.any_stale && (grad->dfinal_state || grad->dinit_state || grad->stage != 0))
    return set_error(TS_ERR_NOT_IMPLEMENTED, "scan_bwd: stale retentions take no boundary states or stages");
  g.dq = grad->dq;
  g.dk = grad->dk;
  g.dv = grad->dv;
  for (int i = 0; i < 3; ++i) g.dvs[i] = grad->dv_strides[i];
  g.dv_strided = (grad->dv_strides[0] | grad->dv_strides[1] | grad->dv_strides[2]) != 0;
  g.grad_bf16 = grad->grad_dtype == TS_DTYPE_BF16;
  if (grad->stage < 0 || grad->stage > 2) return set_error(TS_ERR_VALUE, "scan_bwd: stage must be 0, 1 or 2");
  g.dfinal = grad->dfinal_state;
  g.dinit = grad->dinit_state;
  g.store = 1;
  g.all_tiles = (g.dfinal != nullptr || g.dinit != nullptr || p.init != nullptr || grad->stage != 0) ? 1 : 0;
  g.gstates = static_cast<float*>(grad->workspace);
  g.gimages = reinterpret_cast<__nv_bfloat16*>(static_cast<uint8_t*>(grad->workspace) + states_bytes(p));
  g.pstates = reinterpret_cast<__nv_bfloat16*>(static_cast<uint8_t*>(grad->workspace) + states_bytes(p) + images_bytes(p));
  g.gsegs = reinterpret_cast<float*>(static_cast<uint8_t*>(grad->workspace) + 2 * states_bytes(p) + images_bytes(p));
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (grad->stage == 1) {
    // local tile terms and the gradient of the initial state from this shard's outputs
    if (!g.dinit) return set_error(TS_ERR_VALUE, "scan_bwd: stage 1 needs dinit_state");
    g.dfinal = nullptr;
    g.store = 0;
    return launch_scan_bwd(p, g, s, true, false);
  }
  // stage 2 continues stage 1, whose final state started from zero
  g.zero_start_final = grad->stage == 2;
  return launch_scan_bwd(p, g, s, grad->stage == 0, true);
}

}  // extern "C"
