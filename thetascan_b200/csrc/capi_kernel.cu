// C-ABI entry points of the kernel-family feature and key-mass-read kernels.
#include <cstring>

#include "capi_internal.h"
#include "common.cuh"

namespace ts {

struct FeatParams;
struct ReadParams;
struct MassParams;
int launch_feature_fwd(const FeatParams& p, cudaStream_t s);
int launch_feature_bwd(const FeatParams& p, cudaStream_t s);
size_t feature_fwd_smem(const FeatParams& p);
size_t feature_bwd_smem(const FeatParams& p);
int launch_kread_fwd(const ReadParams& p, cudaStream_t s);
int launch_kread_bwd(const ReadParams& p, cudaStream_t s);
int launch_mass_fwd(const MassParams& p, cudaStream_t s);
int launch_mass_bwd(const MassParams& p, cudaStream_t s);

namespace {
constexpr size_t kMaxSmemBlock = 232448;

int build_feature_params(const ts_feature_args* a, FeatParams* p) {
  if (!a) return set_error(TS_ERR_VALUE, "feature: null arguments");
  if (a->batch < 1 || a->heads < 1 || a->tokens < 1)
    return set_error(TS_ERR_VALUE, "feature: batch, heads and tokens must be >= 1");
  if (a->head_dim < 1 || a->head_dim > 128)
    return set_error(TS_ERR_NOT_IMPLEMENTED, "feature: head_dim %d outside 1..128", a->head_dim);
  if (a->projections < 1 || a->projections > 256)
    return set_error(TS_ERR_NOT_IMPLEMENTED, "feature: %d projections outside 1..256", a->projections);
  if (a->kind < TS_FEATURE_RELU2 || a->kind > TS_FEATURE_BSPLINE)
    return set_error(TS_ERR_VALUE, "feature: unknown kind %d", a->kind);
  if (!a->k || !a->w1 || !a->phi_k) return set_error(TS_ERR_VALUE, "feature: null k, w1 or phi_k");
  if (a->q && !a->phi_q) return set_error(TS_ERR_VALUE, "feature: phi_q is required with q");
  std::memset(p, 0, sizeof(*p));
  p->B = a->batch;
  p->H = a->heads;
  p->T = a->tokens;
  p->d = a->head_dim;
  p->dP = round_up(a->head_dim, 16);
  p->P = a->projections;
  p->PP = round_up(a->projections, 16);
  p->PM = round_up(a->projections, 128);
  p->kind = a->kind;
  p->nb = a->kind == TS_FEATURE_BSPLINE ? a->basis : 1;
  if (a->kind == TS_FEATURE_BSPLINE) {
    if (a->basis < 8 || a->basis > 16 || a->basis % 8)
      return set_error(TS_ERR_NOT_IMPLEMENTED, "feature: B-spline basis count %d must be 8 or 16", a->basis);
    if (!(a->bound > 0.f)) return set_error(TS_ERR_VALUE, "feature: B-spline bound must be positive");
  }
  p->m = p->P * p->nb;
  if (p->m > 256) return set_error(TS_ERR_NOT_IMPLEMENTED, "feature: feature width %d exceeds 256", p->m);
  p->mP = round_up(p->m, 16);
  p->mM = round_up(p->m, 128);
  p->eps = a->eps;
  p->bound = a->bound;
  p->x[0] = static_cast<const __nv_bfloat16*>(a->k);
  p->x[1] = static_cast<const __nv_bfloat16*>(a->q);
  for (int i = 0; i < 3; ++i) {
    p->xs[0][i] = a->k_strides[i];
    p->xs[1][i] = a->q_strides[i];
  }
  p->W1 = static_cast<const __nv_bfloat16*>(a->w1);
  p->W2 = static_cast<const __nv_bfloat16*>(a->w2);
  p->bias = a->score_bias;
  p->thr = a->threshold;
  p->gain = a->gain;
  p->gain_mode = a->gain ? (a->gain_per_feature ? 2 : 1) : 0;
  p->gain_scalar = a->gain_scalar;
  p->scale = a->spline_scale;
  p->scale_scalar = a->spline_scale_scalar;
  p->phi[0] = static_cast<__nv_bfloat16*>(a->phi_k);
  p->phi[1] = static_cast<__nv_bfloat16*>(a->phi_q);
  p->phi_q32 = a->q ? a->phi_q_f32 : nullptr;
  if (p->phi_q32 && (reinterpret_cast<uintptr_t>(p->phi_q32) & 15))
    return set_error(TS_ERR_VALUE, "feature: phi_q_f32 must be 16-byte aligned");
  p->y0 = a->y0;
  p->nsel = a->q ? 2 : 1;
  p->sel0 = 0;
  if (a->rope_rot < 0 || a->rope_rot % 2 || a->rope_rot > a->head_dim)
    return set_error(TS_ERR_VALUE, "feature: rope_rot %d must be even and within 0..head_dim", a->rope_rot);
  if (a->rope_rot > 0 && (!a->rope_cos || !a->rope_sin))
    return set_error(TS_ERR_VALUE, "feature: rope_cos and rope_sin are required with rope_rot");
  if (a->rope_pos0 < 0) return set_error(TS_ERR_VALUE, "feature: rope_pos0 must be >= 0");
  if (a->l2norm && !(a->l2norm_eps > 0.f)) return set_error(TS_ERR_VALUE, "feature: l2norm_eps must be positive");
  p->rot = a->rope_rot;
  p->rcos = a->rope_cos;
  p->rsin = a->rope_sin;
  p->pos0 = a->rope_pos0;
  p->l2norm = a->l2norm ? 1 : 0;
  p->neps = a->l2norm_eps;
  if (a->sparsity < TS_SPARSITY_NONE || a->sparsity > TS_SPARSITY_RELATIVE_ST_BLEND)
    return set_error(TS_ERR_VALUE, "feature: unknown sparsity %d", a->sparsity);
  if (a->sparsity != TS_SPARSITY_NONE) {
    if (a->kind != TS_FEATURE_SOFTMAX)
      return set_error(TS_ERR_VALUE, "feature: relative sparsity is defined for the softmax partition only");
    if (!a->relative_threshold) return set_error(TS_ERR_VALUE, "feature: relative sparsity needs relative_threshold");
    if (a->sparsity == TS_SPARSITY_RELATIVE_ST_BLEND && !a->sparse_blend)
      return set_error(TS_ERR_VALUE, "feature: relative_st_blend needs sparse_blend");
    if (!(a->threshold_temperature > 0.f))
      return set_error(TS_ERR_VALUE, "relative threshold temperature must be positive");
  }
  p->sparse_mode = a->sparsity;
  p->temperature = a->threshold_temperature;
  p->rho = a->relative_threshold;
  p->alpha = a->sparse_blend;
  return TS_OK;
}

int build_read_params(const ts_kread_args* a, ReadParams* p) {
  if (!a) return set_error(TS_ERR_VALUE, "kread: null arguments");
  if (a->batch < 1 || a->heads < 1 || a->tokens < 1 || a->head_dim < 1)
    return set_error(TS_ERR_VALUE, "kread: sizes must be >= 1");
  if (a->mode < TS_VIEWS_SUM || a->mode > TS_VIEWS_STALE) return set_error(TS_ERR_VALUE, "kread: unknown mode");
  const int J = a->mode == TS_VIEWS_SUM ? 0 : a->branches;
  if (J < 0 || J > TS_MAX_RETENTIONS - 1)
    return set_error(TS_ERR_NOT_IMPLEMENTED, "kread: %d recency branches (at most %d)", J, TS_MAX_RETENTIONS - 1);
  if (a->mode != TS_VIEWS_SUM && J < 1) return set_error(TS_ERR_VALUE, "kread: a bank needs >= 1 branch");
  if (J > 0 && !a->eta) return set_error(TS_ERR_VALUE, "kread: eta is required with recency branches");
  for (int s = 0; s <= J; ++s)
    if (!a->slots[s]) return set_error(TS_ERR_VALUE, "kread: null slot %d", s);
  if (!a->y0) return set_error(TS_ERR_VALUE, "kread: null y0");
  std::memset(p, 0, sizeof(*p));
  p->B = a->batch;
  p->H = a->heads;
  p->T = a->tokens;
  p->d = a->head_dim;
  p->J = J;
  p->mode = a->mode;
  p->eps = a->eps;
  if (a->mass_columns < 0 || a->mass_columns > 2)
    return set_error(TS_ERR_VALUE, "kread: mass_columns must be 1 or 2 (0 = 1)");
  p->mass_cols = a->unnormalized ? 0 : a->mass_columns == 2 ? 2 : 1;
  for (int s = 0; s <= J; ++s) p->out[s] = a->slots[s];
  p->eta = a->eta;
  p->y0 = a->y0;
  p->y = static_cast<__nv_bfloat16*>(a->y);
  return TS_OK;
}
int build_mass_params(const ts_mass_args* a, MassParams* p) {
  if (!a) return set_error(TS_ERR_VALUE, "mass: null arguments");
  if (a->batch < 1 || a->heads < 1 || a->tokens < 1) return set_error(TS_ERR_VALUE, "mass: sizes must be >= 1");
  if (a->width < 2 || a->width > 512 || (a->width & 1))
    return set_error(TS_ERR_NOT_IMPLEMENTED, "mass: feature width %d must be even and in 2..512", a->width);
  if (!a->phi_k || (!a->phi_q && !a->phi_q_f32)) return set_error(TS_ERR_VALUE, "mass: null phi_k or phi_q");
  if (a->stale && !a->log_alpha) return set_error(TS_ERR_VALUE, "mass: the stale mass needs a log_alpha");
  if ((reinterpret_cast<uintptr_t>(a->phi_k) | reinterpret_cast<uintptr_t>(a->phi_q)) & 3)
    return set_error(TS_ERR_VALUE, "mass: phi_k and phi_q must be 4-byte aligned");
  std::memset(p, 0, sizeof(*p));
  p->B = a->batch;
  p->H = a->heads;
  p->T = a->tokens;
  p->m = a->width;
  p->phi_k = static_cast<const __nv_bfloat16*>(a->phi_k);
  p->phi_q32 = a->phi_q_f32;
  if (reinterpret_cast<uintptr_t>(a->phi_q_f32) & 7) return set_error(TS_ERR_VALUE, "mass: phi_q_f32 must be 8-byte aligned");
  p->phi_q = static_cast<const __nv_bfloat16*>(a->phi_q);
  p->la = a->log_alpha;
  p->stale = a->stale ? 1 : 0;
  p->eps = a->eps;
  p->qs = a->q_scaled;
  p->qs_f32 = a->q_scaled_f32 ? 1 : 0;
  if (p->qs_f32 && (reinterpret_cast<uintptr_t>(a->q_scaled) & 7))
    return set_error(TS_ERR_VALUE, "mass: an f32 q_scaled must be 8-byte aligned");
  return TS_OK;
}
}  // namespace

}  // namespace ts

using namespace ts;

extern "C" {

int ts_b200_feature_fwd(const ts_feature_args* args, ts_stream_t stream) {
  FeatParams p;
  if (int e = build_feature_params(args, &p)) return e;
  if (feature_fwd_smem(p) > kMaxSmemBlock)
    return set_error(TS_ERR_NOT_IMPLEMENTED, "feature: shapes exceed the shared-memory budget of one CTA");
  return launch_feature_fwd(p, reinterpret_cast<cudaStream_t>(stream));
}

int ts_b200_feature_bwd(const ts_feature_args* args, const ts_feature_grad_args* grad, ts_stream_t stream) {
  FeatParams p;
  if (int e = build_feature_params(args, &p)) return e;
  if (!grad || !grad->dphi_k || !grad->dw1) return set_error(TS_ERR_VALUE, "feature_bwd: dphi_k and dw1 are required");
  if ((grad->dk == nullptr) == (grad->dk_bf16 == nullptr))
    return set_error(TS_ERR_VALUE, "feature_bwd: exactly one of dk and dk_bf16 is required");
  if (args->q && (!grad->dphi_q || (grad->dq == nullptr) == (grad->dq_bf16 == nullptr)))
    return set_error(TS_ERR_VALUE, "feature_bwd: dphi_q and exactly one of dq and dq_bf16 are required");
  if (feature_bwd_smem(p) > kMaxSmemBlock)
    return set_error(TS_ERR_NOT_IMPLEMENTED, "feature_bwd: shapes exceed the shared-memory budget of one CTA");
  p.dphi[0] = grad->dphi_k;
  p.dphi[1] = grad->dphi_q;
  p.dphi_bf16 = grad->dphi_dtype == TS_DTYPE_BF16;
  p.dy = grad->dy0;
  p.dyb = static_cast<const __nv_bfloat16*>(grad->dy0_bf16);
  for (int i = 0; i < 3; ++i) p.dys[i] = grad->dy0_strides[i];
  if (p.dy && p.dyb) return set_error(TS_ERR_VALUE, "feature_bwd: give at most one of dy0 and dy0_bf16");
  p.dx[0] = grad->dk;
  p.dx[1] = grad->dq;
  p.dxb[0] = static_cast<__nv_bfloat16*>(grad->dk_bf16);
  p.dxb[1] = static_cast<__nv_bfloat16*>(grad->dq_bf16);
  for (int i = 0; i < 3; ++i) {
    p.dxs[0][i] = grad->dk_strides[i];
    p.dxs[1][i] = grad->dq_strides[i];
  }
  p.dW1 = grad->dw1;
  p.dW2_t = grad->dw2_transposed ? 1 : 0;
  p.dW2 = grad->dw2;
  p.dbias = grad->dscore_bias;
  p.dthr = grad->dthreshold;
  p.dgain = grad->dgain;
  p.dscale = grad->dspline_scale;
  p.drho = grad->drelative_threshold;
  p.dalpha = grad->dsparse_blend;
  return launch_feature_bwd(p, reinterpret_cast<cudaStream_t>(stream));
}

int ts_b200_kread_fwd(const ts_kread_args* args, ts_stream_t stream) {
  ReadParams p;
  if (int e = build_read_params(args, &p)) return e;
  if (!args->y) return set_error(TS_ERR_VALUE, "kread: null y");
  return launch_kread_fwd(p, reinterpret_cast<cudaStream_t>(stream));
}

int ts_b200_kread_bwd(const ts_kread_args* args, const ts_kread_grad_args* grad, ts_stream_t stream) {
  ReadParams p;
  if (int e = build_read_params(args, &p)) return e;
  if (!grad || !grad->dy) return set_error(TS_ERR_VALUE, "kread_bwd: dy is required");
  for (int s = 0; s <= p.J; ++s)
    if (!grad->dslots[s]) return set_error(TS_ERR_VALUE, "kread_bwd: null dslot %d", s);
  p.dy = grad->dy;
  p.dy_bf16 = grad->dy_dtype == TS_DTYPE_BF16;
  for (int s = 0; s <= p.J; ++s) p.dout[s] = static_cast<__nv_bfloat16*>(grad->dslots[s]);
  p.dy0 = grad->dy0;
  p.deta = grad->deta;
  return launch_kread_bwd(p, reinterpret_cast<cudaStream_t>(stream));
}

int ts_b200_mass_query_fwd(const ts_mass_args* args, ts_stream_t stream) {
  MassParams p;
  if (int e = build_mass_params(args, &p)) return e;
  if (!p.qs) return set_error(TS_ERR_VALUE, "mass: null q_scaled");
  return launch_mass_fwd(p, reinterpret_cast<cudaStream_t>(stream));
}

size_t ts_b200_mass_query_bwd_workspace_bytes(const ts_mass_args* args) {
  MassParams p;
  if (build_mass_params(args, &p) != TS_OK) return 0;
  return static_cast<size_t>(p.B) * p.H * p.T * p.m * sizeof(float);
}

int ts_b200_mass_query_bwd(const ts_mass_args* args, const ts_mass_grad_args* grad, ts_stream_t stream) {
  MassParams p;
  if (int e = build_mass_params(args, &p)) return e;
  if (!grad || !grad->dq_scaled || !grad->dphi_q || !grad->dphi_k)
    return set_error(TS_ERR_VALUE, "mass_bwd: dq_scaled, dphi_q and dphi_k are required");
  const size_t need = static_cast<size_t>(p.B) * p.H * p.T * p.m * sizeof(float);
  if (!grad->workspace || grad->workspace_bytes < need)
    return set_error(TS_ERR_VALUE, "mass_bwd: workspace of %zu bytes needed", need);
  if (((reinterpret_cast<uintptr_t>(grad->dphi_q) | reinterpret_cast<uintptr_t>(grad->dphi_k) |
        reinterpret_cast<uintptr_t>(grad->workspace)) & 7) ||
      (reinterpret_cast<uintptr_t>(grad->dq_scaled) & (grad->dq_dtype == TS_DTYPE_BF16 ? 3 : 7)))
    return set_error(TS_ERR_VALUE, "mass_bwd: misaligned gradient buffers");
  p.dqs = grad->dq_scaled;
  p.dqs_bf16 = grad->dq_dtype == TS_DTYPE_BF16;
  p.dphi_q = grad->dphi_q;
  p.dphi_k = grad->dphi_k;
  p.dla = grad->dlog_alpha;
  p.dmass = static_cast<float*>(grad->workspace);
  return launch_mass_bwd(p, reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"

// ---------------------------------------------------------------- GN rows

int ts_b200_gn_rows(const ts_gn_rows_args* a, ts_stream_t stream) {
  using namespace ts;
  if (!a) return set_error(TS_ERR_VALUE, "gn_rows: null arguments");
  if (a->batch < 0 || a->heads < 0 || a->tokens < 0)
    return set_error(TS_ERR_VALUE, "gn_rows: negative shape");
  if (a->d < 1 || a->m < 1 || a->d > kGnMaxWidth || a->m > kGnMaxWidth)
    return set_error(TS_ERR_NOT_IMPLEMENTED, "gn_rows: widths d=%d, m=%d outside 1..%d", a->d, a->m, kGnMaxWidth);
  if (a->nonlinearity < TS_GN_RELU2 || a->nonlinearity > TS_GN_TANH)
    return set_error(TS_ERR_NOT_IMPLEMENTED, "gn_rows: unknown nonlinearity %d", a->nonlinearity);
  // inputs and outputs each stage needs (1 = required, 2 = optional)
  static const char kIn[13][9] = {
      "", "11", "111111", "11", "1", "12", "111", "11", "121", "11", "11", "11111111", "1111111"};
  static const char kOut[13][5] = {"", "1111", "1", "1", "1", "1", "1", "1", "12", "1", "1", "1111", "1"};
  if (a->stage < TS_GN_WRITE_PRE || a->stage > TS_GN_WRITE_PRE_BWD)
    return set_error(TS_ERR_VALUE, "gn_rows: unknown stage %d", a->stage);
  for (int i = 0; kIn[a->stage][i]; ++i)
    if (kIn[a->stage][i] == '1' && !a->in[i]) return set_error(TS_ERR_VALUE, "gn_rows: stage %d needs in[%d]", a->stage, i);
  const bool bf16_only = (a->stage == TS_GN_WRITE_G || a->stage == TS_GN_QUERY_PRE) && a->out_bf16;
  for (int i = 0; kOut[a->stage][i]; ++i)
    if (kOut[a->stage][i] == '1' && !a->out[i] && !(i == 0 && bf16_only))
      return set_error(TS_ERR_VALUE, "gn_rows: stage %d needs out[%d]", a->stage, i);
  if (a->out_bf16 && a->stage > TS_GN_FEATURES)
    return set_error(TS_ERR_VALUE, "gn_rows: out_bf16 is for the forward stages WRITE_PRE .. FEATURES");
  if (a->stage == TS_GN_FEATURES_BWD && a->in[1] && !a->out[1])
    return set_error(TS_ERR_VALUE, "gn_rows: a read's gradient needs out[1]");
  if (a->stage == TS_GN_OUT_BWD && !(a->flags & 1))
    return set_error(TS_ERR_VALUE, "gn_rows: OUT_BWD is the normalised read's (flags bit 0)");
  GnRowParams p{};
  p.B = a->batch;
  p.H = a->heads;
  p.T = a->tokens;
  p.d = a->d;
  p.m = a->m;
  p.nonlin = a->nonlinearity;
  p.flags = a->flags;
  p.eps = a->eps;
  p.tau = a->tau;
  p.dtau = a->tau ? a->dtau : nullptr;
  for (int i = 0; i < 8; ++i) p.in[i] = a->in[i];
  for (int i = 0; i < 4; ++i) p.out[i] = a->out[i];
  p.out_bf16 = static_cast<__nv_bfloat16*>(a->out_bf16);
  return launch_gn_rows(p, a->stage, reinterpret_cast<cudaStream_t>(stream));
}

static int build_gn_prep(const ts_gn_prep_args* a, ts::GnPrepParams* p, bool backward) {
  using namespace ts;
  if (!a) return set_error(TS_ERR_VALUE, "gn_prep: null arguments");
  if (a->batch < 0 || a->heads < 0 || a->tokens < 0) return set_error(TS_ERR_VALUE, "gn_prep: negative shape");
  if (a->d < 1 || a->d > kGnMaxWidth) return set_error(TS_ERR_NOT_IMPLEMENTED, "gn_prep: d=%d outside 1..256", a->d);
  if (a->rot < 0 || a->rot > a->d || (a->rot & 1))
    return set_error(TS_ERR_VALUE, "gn_prep: rot=%d must be even and <= d", a->rot);
  if (a->rot && (!a->cos || !a->sin)) return set_error(TS_ERR_VALUE, "gn_prep: null phase tables");
  if (!a->qkv) return set_error(TS_ERR_VALUE, "gn_prep: null qkv");
  if (backward ? (!a->dq || !a->dk || !a->dv || !a->dqkv) : (!a->q || !a->k || !a->v))
    return set_error(TS_ERR_VALUE, "gn_prep: null stream pointer");
  *p = GnPrepParams{a->batch, a->heads, a->tokens, a->d, a->rot, a->eps, a->qkv, a->cos, a->sin,
                    a->q, a->k, a->v, a->dq, a->dk, a->dv, a->dqkv};
  return TS_OK;
}

int ts_b200_gn_prep_fwd(const ts_gn_prep_args* a, ts_stream_t stream) {
  ts::GnPrepParams p;
  if (int e = build_gn_prep(a, &p, false)) return e;
  return ts::launch_gn_prep(p, false, reinterpret_cast<cudaStream_t>(stream));
}

int ts_b200_gn_prep_bwd(const ts_gn_prep_args* a, ts_stream_t stream) {
  ts::GnPrepParams p;
  if (int e = build_gn_prep(a, &p, true)) return e;
  return ts::launch_gn_prep(p, true, reinterpret_cast<cudaStream_t>(stream));
}
