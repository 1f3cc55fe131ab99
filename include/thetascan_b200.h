/*
 * thetascan_b200 -- C ABI of the B200 (sm_100a) ThetaScan hot path.
 *
 * The reference ThetaScan v0.1.0 is pure PyTorch and has no foreign-function
 * boundary; each entry point below names the reference interface it stands in
 * for (paths relative to the reference project root).  A Python host reaches
 * these through ctypes (thetascan_b200/_lib.py); any other host binds them the
 * same way, with plain pointers, sizes and this header's structs.
 *
 * Conventions
 *  - All tensor pointers are DEVICE pointers on the current CUDA device.
 *  - Work is enqueued on the caller's stream; no entry point synchronizes
 *    except ts_b200_device_status.
 *  - The library allocates no device memory: outputs and workspaces are
 *    caller-allocated; ts_b200_*_workspace_bytes report the sizes.
 *  - Return value: TS_OK (0) or one of the TS_ERR_* codes; the message of the
 *    last failure on the calling thread is available from ts_b200_last_error.
 *    TS_ERR_VALUE corresponds to the reference's ValueError (bad shape or
 *    argument), TS_ERR_NOT_IMPLEMENTED to NotImplementedError, TS_ERR_CUDA to
 *    a RuntimeError from the CUDA runtime.
 *  - Kernels never trap and never wait without bound: a bounded wait that
 *    gives up records a nonzero device status, read by ts_b200_device_status.
 */
#ifndef THETASCAN_B200_H_
#define THETASCAN_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* ts_stream_t; /* == cudaStream_t */

enum {
  TS_OK = 0,
  TS_ERR_VALUE = 1,
  TS_ERR_NOT_IMPLEMENTED = 2,
  TS_ERR_CUDA = 3,
  TS_ERR_DEVICE = 4
};

enum { TS_DTYPE_F32 = 0, TS_DTYPE_BF16 = 1 };

#define TS_MAX_RETENTIONS 4

/* ------------------------------------------------------------------ misc */

/* Library version string. */
const char* ts_b200_version(void);

/* Kernels this library has launched in the process so far (every entry
 * point counts each of its launches).  No reference counterpart: a host
 * reads it before and after a region to count the region's launches. */
long long ts_b200_launch_count(void);

/* Copy the message of the last failed call on this thread into buf (always
 * NUL-terminated); returns that call's error code. */
int ts_b200_last_error(char* buf, size_t len);

/* Synchronize `stream`, then read and clear the device status word written
 * by bounded waits that gave up (0 = healthy).  Returns TS_ERR_DEVICE if it
 * was nonzero, TS_ERR_CUDA if the synchronization failed. */
int ts_b200_device_status(ts_stream_t stream, int* status);

/* Tensor-core self-test: D[128 x N] (f32) = A[128 x K] . B[K x N] (bf16,
 * row-major), with A staged MN-major if a_mn and B staged MN-major if b_mn.
 * No reference counterpart: it validates the tcgen05 operand layouts. */
int ts_b200_selftest_mma(const void* A, const void* B, float* D, int N, int K, int a_mn, int b_mn,
                         ts_stream_t stream);

/* The same product with both operands loaded by TMA (64-column boxes, 128-byte
 * swizzle) and read through swizzled descriptors.  Sources: A [128 x K]
 * row-major, or A^T [K x 128] if a_mn; B [K x N] row-major if b_mn, else
 * B^T [N x K].  N and K are 64 or 128.  No reference counterpart: it
 * validates the operand layouts of the TMA-fed kernels. */
int ts_b200_selftest_tma_mma(const void* A, const void* B, float* D, int N, int K, int a_mn, int b_mn,
                             ts_stream_t stream);

/* ------------------------------------------------------------------ scan
 *
 * Multi-view inclusive causal scan, the contract of
 *   scan_chunk.linattn_views(q, k, v, retentions, chunk)
 *   (src/thetascan/_core/ops/scan_chunk.py:246-339)
 * out_r[t] = sum_{i<=t} w_r(t,i) (q_t . k_i) v_i  for every retention r, with
 * w = 1 (plain sum), alpha_h^(t-i) (static per-head log-retention) or
 * 1 - alpha_h^(t-i) (the stale view, `stale` below).  The
 * score tile q.k^T is formed once and shared by all retentions; the carried
 * state is f32.  Streams are bf16 (f32 with f32_streams below); their
 * innermost dimension is contiguous.
 */
typedef struct ts_scan_args {
  int batch, heads, tokens;
  int dk;               /* key/query width, 1..256 */
  int dv;               /* payload width incl. the unit column if v_append_unit, 1..256 (within the CTA budgets) */
  const void* q;        /* bf16 [B,H,T,dk] */
  const void* k;        /* bf16 [B,H,T,dk] */
  const void* v;        /* bf16 [B,H,T,dv - v_append_unit] */
  int64_t q_strides[3]; /* element strides of batch, head, token */
  int64_t k_strides[3];
  int64_t v_strides[3];
  int v_append_unit;    /* 1: the payload is [v | 1] (key-mass read, engine.py:430);
                         * 2: [v | 1 | 1], the mass column twice, so that a read
                         * gradient can hand its mass part over as bf16 hi + lo */
  int n_retentions;     /* 1..TS_MAX_RETENTIONS */
  /* NULL = plain causal sum; else device f32 [heads] static log-retention */
  const float* log_alpha[TS_MAX_RETENTIONS];
  void* out[TS_MAX_RETENTIONS]; /* [B,H,T,dv] contiguous, out_dtype */
  int out_dtype;                /* TS_DTYPE_F32 or TS_DTYPE_BF16 */
  /* Caller-owned scratch of ts_b200_scan_workspace_bytes(args) bytes.  After
   * ts_b200_scan_fwd it holds the carried chunk states that the backward
   * reads, so keep it unchanged between the two calls. */
  void* workspace;
  size_t workspace_bytes;
  /* Optional boundary states of a sequence shard, f32 [B,H,R,dk,dv]
   * (feature-major, payload column fastest; R = n_retentions):
   *   init_state  the state entering token 0 (NULL = zero state);
   *   final_state receives the state after the last token (NULL = not written).
   * `stage` splits the forward around an exchange of shard states:
   *   0  whole forward (init_state used, final_state written if given);
   *   1  tile states of every tile and final_state from a ZERO initial state,
   *      no outputs (final_state required);
   *   2  the rest of the forward from init_state: carried states and the
   *      outputs, reusing the tile states that stage 1 left in the workspace
   *      (same workspace, same inputs).
   * Sequence parallelism: stage 1 on every shard, exchange the final states,
   * compose each shard's entering state, stage 2 on every shard. */
  const float* init_state;
  float* final_state;
  int stage;
  /* stale[r] != 0: retention r reads the STALE view of log_alpha[r], weights
   * 1 - alpha_h^(t-i) (zero for the current token), which is the reference's
   * FadeStale view S_sum - S_fast (src/thetascan/_core/ops/interface.py:
   * 251-279) formed without the cancellation of that difference.  Needs
   * log_alpha[r]; takes no boundary states (init/final NULL, stage 0).  Each
   * stale retention carries one extra decayed state in the workspace. */
  int stale[TS_MAX_RETENTIONS];
  /* Nonzero: q, k, v are f32 streams, out is f32 (out_dtype TS_DTYPE_F32),
   * and the backward's dout, dq, dk and dv are f32 (grad_dtype TS_DTYPE_F32,
   * dv contiguous).  Float32 streams are scanned with f32 FMAs on the CUDA
   * cores -- bf16 or tf32 tensor-core operands cannot meet the reference's
   * float32 tolerance (rel-err 1e-5) -- for dk, dv <= 256 within the shared
   * memory of one CTA (dk 128 with dv up to 248, dk 256 with dv up to 123), without
   * stale retentions, boundary states or stages (TS_ERR_NOT_IMPLEMENTED
   * otherwise; a stale view of f32 streams is the difference of the plain and
   * recency reads, which the host forms as the reference does).  Zero: bf16
   * streams on the tensor cores. */
  int f32_streams;
  /* Per-token retention streams, the [B,H,T,1] decay of the reference's
   * chunk scan (scan_chunk.py:122-155, 208-212; the data-dependent EMA views
   * of interface.py:216-230): where log_alpha_stream[r] is non-NULL it is a
   * contiguous f32 [B,H,T] log-retention stream (<= 0) and retention r reads
   * with w(t,i) = exp(sum_{i<s<=t} log_alpha_stream[s]) in place of
   * log_alpha[r] (which must then be NULL).  f32 streams only
   * (TS_ERR_NOT_IMPLEMENTED otherwise); the backward writes
   * ts_scan_grad_args.dlog_alpha_stream[r]. */
  const float* log_alpha_stream[TS_MAX_RETENTIONS];
} ts_scan_args;

size_t ts_b200_scan_workspace_bytes(const ts_scan_args* args);

/* Forward of the multi-view scan (scan_chunk.py:246-339). */
int ts_b200_scan_fwd(const ts_scan_args* args, ts_stream_t stream);

/* Gradients of the multi-view scan (the autograd of scan_chunk.py:246-339,
 * pinned by tests/test_scan_chunk.py:271-340 of the reference).
 * dout[r]: bf16 [B,H,T,dv] contiguous (f32 for f32 streams).  dq/dk f32 or
 * bf16 [B,H,T,dk], dv
 * [B,H,T,dv] contiguous in grad_dtype (dv excludes nothing: with
 * v_append_unit the unit column's gradient is computed and discarded).
 * dlog_alpha[r]: device f32 [heads], ACCUMULATED into (zero it first); may be
 * NULL for plain-sum retentions. */
typedef struct ts_scan_grad_args {
  const void* dout[TS_MAX_RETENTIONS];
  void* dq;
  void* dk;
  void* dv;
  int grad_dtype;
  float* dlog_alpha[TS_MAX_RETENTIONS];
  void* workspace; /* ts_b200_scan_bwd_workspace_bytes(fwd) bytes */
  size_t workspace_bytes;
  /* All zero: dv is contiguous [B,H,T,dv].  Otherwise element strides
   * (batch, head, token) of a [B,H,T,dv - v_append_unit] view that receives
   * the payload gradient (the unit column's gradient is not written), for
   * instance the v slot of the gradient of a fused qkv projection. */
  int64_t dv_strides[3];
  /* Boundary gradients of a sequence shard (f32 [B,H,R,dk,dv]), and the
   * backward split around their exchange:
   *   dfinal_state gradient of the forward's final_state (NULL = zero);
   *   dinit_state  receives the gradient of init_state (NULL = not written);
   *   stage 0  whole backward;
   *        1  local tile terms of every tile and dinit_state of the shard's own
   *           outputs (dinit_state required; nothing else is written except the
   *           log-retention terms of this stage);
   *        2  the rest from dfinal_state, the gradient of stage 1's final
   *           state (the zero-start total): dq, dk, dv and the remaining
   *           log-retention terms (same workspaces as stage 1). */
  const float* dfinal_state;
  float* dinit_state;
  int stage;
  /* Gradients of the per-token retention streams, f32 [B,H,T] (written, not
   * accumulated), or NULL (not wanted). */
  float* dlog_alpha_stream[TS_MAX_RETENTIONS];
} ts_scan_grad_args;

size_t ts_b200_scan_bwd_workspace_bytes(const ts_scan_args* fwd);
int ts_b200_scan_bwd(const ts_scan_args* fwd, const ts_scan_grad_args* grad, ts_stream_t stream);

/* Forward of the multi-view scan without any caller workspace.  No
 * counterpart in the reference: it exists for hosts that cannot allocate
 * device memory for this library -- a runtime whose allocator owns all device
 * memory and lends none to plug-ins, or a serving loop that forbids cudaMalloc
 * once it is running.  Same inputs, outputs and results as ts_b200_scan_fwd;
 * args->workspace and args->workspace_bytes are ignored.
 *  - Scratch is one fixed device array of TS_STATIC_SCRATCH_BYTES inside the
 *    library, held by every GPU that loads it until the process exits.  A
 *    shape needing more (ts_b200_scan_workspace_bytes > the limit) is
 *    rejected with TS_ERR_VALUE before anything is launched.
 *  - Every call looks up the array's device address in the current device's
 *    context (a host-side lookup, no stream operation), so the address stays
 *    right after that context is destroyed and created again.  The first
 *    lookup on a device may load the library's module there: make the first
 *    call on each device before any stream capture.
 *  - All calls on one GPU share that GPU's copy of the array, which keeps
 *    the last call's contents: calls that overlap on the same GPU (say, on
 *    two streams) race, so serialize them.  Nothing in it needs clearing:
 *    each call writes every scratch element before reading it.
 *  - Forward only: the chunk states are not kept for ts_b200_scan_bwd. */
#define TS_STATIC_SCRATCH_BYTES (16u << 20)
int ts_b200_scan_fwd_static(const ts_scan_args* args, ts_stream_t stream);


/* ------------------------------------------------------------------ feature maps
 *
 * Kernel-family write/read features, per token and head:
 *   a = W1 x, pre = RMSNorm(a), phi = map(pre)
 * for x = k (write keys) and x = q (read queries), and for q also the slow
 * decode plus residual y0 = q + W2 phi(q).  Stands in for the feature chain of
 *   engine._block_forward / dual_read_views.features
 *   (src/thetascan/_core/ops/engine.py:117-158, 369-395, 522-526),
 *   norms.rmsnorm (src/thetascan/_core/modules/norms.py:5-8) and
 *   kernel_features.feature_map (src/thetascan/_core/ops/kernel_features.py:233-273).
 */
enum { TS_FEATURE_RELU2 = 0, TS_FEATURE_SOFTMAX = 1, TS_FEATURE_BSPLINE = 2 };

typedef struct ts_feature_args {
  int batch, heads, tokens;
  int head_dim;             /* d, 1..128 */
  int projections;          /* P = rows of W1, 1..256 */
  int kind;                 /* TS_FEATURE_* */
  int basis;                /* B-spline basis count per projection (multiple of 8, <= 16) */
  float bound;              /* B-spline coordinate bound */
  float eps;                /* RMSNorm / relu2 mass epsilon (core config eps) */
  const void* k;            /* bf16 [B,H,T,d] */
  const void* q;            /* bf16 [B,H,T,d] or NULL */
  int64_t k_strides[3];
  int64_t q_strides[3];
  const void* w1;           /* bf16 [H, P, d] effective (expanded) projection, contiguous */
  const void* w2;           /* bf16 [H, d, m] effective decode, contiguous, or NULL */
  const float* score_bias;  /* f32 [H, m] or NULL (relu2 / softmax) */
  const float* threshold;   /* f32 [H] or NULL (relu2) */
  const float* gain;        /* f32 [H] or [H, m] or NULL (softmax) */
  int gain_per_feature;     /* 1: gain is [H, m] */
  float gain_scalar;        /* used when gain is NULL */
  const float* spline_scale; /* f32 [H] or NULL (B-spline) */
  float spline_scale_scalar;
  void* phi_k;              /* bf16 [B,H,T,m] out */
  void* phi_q;              /* bf16 [B,H,T,m] out (if q) */
  float* y0;                /* f32 [B,H,T,d] out: q + W2 phi(q) (if q and w2), or NULL */
  /* Optional fused prologue; all zero = k and q rows are used as given.
   * Otherwise k and q are the RAW projections: each row is rotated (channel
   * pairs (2i, 2i+1), i < rope_rot/2, by the f32 tables rope_cos / rope_sin
   * [rope_pos0 + tokens, rope_rot/2] at row rope_pos0 + t) and, with l2norm,
   * divided by max(||row||_2, l2norm_eps), in f32, then rounded to bf16:
   * reference rope.py:57-72 (apply_rope) then norms.py:11-12 (l2norm), as
   * block.py:595-599 applies them to q and k.  y0 is then qhat + W2 phi(qhat),
   * and the backward returns gradients of the raw rows. */
  int rope_rot;             /* even, <= head_dim; 0 = no rotation */
  const float* rope_cos;
  const float* rope_sin;
  int rope_pos0;            /* sequence position of token 0 (sequence shards) */
  int l2norm;               /* 1 = L2-normalize each row after the rotation */
  float l2norm_eps;
  /* Optional f32 [B,H,T,m] copy of phi(q) before its bf16 rounding (16-byte
   * aligned), for the feature-mass read, which divides it by the key mass. */
  float* phi_q_f32;
  /* Relative sparsity of the softmax partition (kernel_features.py:43-70,
   * 95-113 of the reference): with logits l = gain (pre + bias), a feature is
   * kept where l_j - max(l) >= log rho_h (rho clamped to [eps, 1 - eps]):
   *   relative_soft      sparse_j = e^{l_j - max} s_j / max(sum_k e^{l_k - max} s_k, eps),
   *                      s = sigmoid((l - max - log rho) / threshold_temperature);
   *   relative_st        the same with the hard gate [margin >= 0] forward and
   *                      the sigmoid's derivative backward;
   *   relative_st_blend  phi = dense + alpha_h (sparse - dense), dense the softmax.
   * TS_SPARSITY_NONE: the softmax partition as is. */
  int sparsity;
  float threshold_temperature;
  const float* relative_threshold;  /* f32 [H]: rho in (0, 1) */
  const float* sparse_blend;        /* f32 [H]: alpha (relative_st_blend) */
} ts_feature_args;

enum {
  TS_SPARSITY_NONE = 0,
  TS_SPARSITY_RELATIVE_SOFT = 1,
  TS_SPARSITY_RELATIVE_ST = 2,
  TS_SPARSITY_RELATIVE_ST_BLEND = 3
};

int ts_b200_feature_fwd(const ts_feature_args* args, ts_stream_t stream);

typedef struct ts_feature_grad_args {
  const void* dphi_k;       /* [B,H,T,m] (grad_dtype of dphi_dtype) */
  const void* dphi_q;       /* [B,H,T,m] or NULL */
  int dphi_dtype;           /* TS_DTYPE_F32 or TS_DTYPE_BF16 */
  const float* dy0;         /* f32 [B,H,T,d] gradient of y0, or NULL */
  float* dk;                /* f32 [B,H,T,d] out */
  float* dq;                /* f32 [B,H,T,d] out (includes dy0 through the residual) */
  float* dw1;               /* f32 [H,P,d], ACCUMULATED */
  float* dw2;               /* f32 [H,d,m], ACCUMULATED, or NULL */
  float* dscore_bias;       /* f32 [H,m], ACCUMULATED, or NULL */
  float* dthreshold;        /* f32 [H], ACCUMULATED, or NULL */
  float* dgain;             /* f32 like gain, ACCUMULATED, or NULL */
  float* dspline_scale;     /* f32 [H], ACCUMULATED, or NULL */
  /* Optional bf16 outputs of the row gradients in place of dk / dq (which are
   * then NULL): element strides (batch, head, token) of [B,H,T,d] views, for
   * instance the k and q slots of the gradient of a fused qkv projection. */
  void* dk_bf16;
  void* dq_bf16;
  int64_t dk_strides[3];
  int64_t dq_strides[3];
  /* Optional bf16 gradient of y0 in place of dy0 (which is then NULL):
   * element strides (batch, head, token) of a [B,H,T,d] view, for instance the
   * token-major gradient of the read output, whose y0 part is the identity. */
  const void* dy0_bf16;
  int64_t dy0_strides[3];
  /* 1: dw2 is f32 [H,m,d] (the transpose of W2's layout), accumulated with
   * vector atomics; 0: [H,d,m].  The backward rebuilds phi(q) for dw2 from
   * q (ts_feature_args.phi_q is not read by it). */
  int dw2_transposed;
  float* drelative_threshold;  /* f32 [H], ACCUMULATED, or NULL (relative sparsity) */
  float* dsparse_blend;        /* f32 [H], ACCUMULATED, or NULL (relative_st_blend) */
} ts_feature_grad_args;

int ts_b200_feature_bwd(const ts_feature_args* args, const ts_feature_grad_args* grad, ts_stream_t stream);

/* ------------------------------------------------------------------ key-mass read
 *
 * Normalized read and temporal-view blend of the kernel family: from the
 * augmented scan reads [N_s | D_s] of every retention slot (slot 0 = plain
 * sum, slot 1+j = recency branch j: its decayed scan for a fast bank, its
 * stale scan, ts_scan_args.stale, for a stale bank) compute
 *   y = y0 + sum_views c_view N_view / (D_view + eps)
 * for the plain sum, a fast bank (c = 1 - sum eta, eta_j) or a stale bank
 * (c = 1, -eta_j; the zero-memory base read it subtracts is y0).  Stands in for
 *   engine.dual_read_views.memory key_mass (src/thetascan/_core/ops/engine.py:419-442)
 *   and ThetaScan.forward.read_with_temporal (src/thetascan/_core/modules/block.py:667-718).
 * y is written token-major, [B,T,H,d], ready for the output gate/projection.
 */
enum { TS_VIEWS_SUM = 0, TS_VIEWS_FAST = 1, TS_VIEWS_STALE = 2 };

typedef struct ts_kread_args {
  int batch, heads, tokens, head_dim;
  int mode;                 /* TS_VIEWS_* */
  int branches;             /* J recency branches, 0..TS_MAX_RETENTIONS-1 */
  float eps;
  const float* slots[TS_MAX_RETENTIONS]; /* f32 [B,H,T,d+mass_columns] */
  const float* eta;         /* f32 [J,H] blend (after any tanh), or NULL if J == 0 */
  const float* y0;          /* f32 [B,H,T,d] */
  void* y;                  /* bf16 [B,T,H,d] out */
  /* Mass columns after the d value columns of every slot: 1 ([N | D], a scan
   * with v_append_unit = 1) or 2 ([N | D | D], v_append_unit = 2); 0 means 1.
   * The backward writes the mass gradient into them (with 2: as bf16 hi + lo),
   * formed from the bf16-rounded value gradient so that the quotient rule's
   * cancellation survives the bf16 hand-over to the scan backward. */
  int mass_columns;
  /* Nonzero: unnormalized blend, mem(s) = N_s, slots f32 [B,H,T,d] (no mass
   * column): the unnormalized read (engine.py:402-416) and the feature-mass
   * read (engine.py:443-456), whose normalization happened on the query side
   * (ts_b200_mass_query_fwd).  mass_columns is then ignored. */
  int unnormalized;
} ts_kread_args;

int ts_b200_kread_fwd(const ts_kread_args* args, ts_stream_t stream);

typedef struct ts_kread_grad_args {
  const void* dy;           /* [B,T,H,d] */
  int dy_dtype;             /* TS_DTYPE_F32 or TS_DTYPE_BF16 */
  void* dslots[TS_MAX_RETENTIONS]; /* bf16 [B,H,T,d+mass_columns] out: gradients of the scan reads */
  float* dy0;               /* f32 [B,H,T,d] out (a copy of dy, head-major), or NULL */
  float* deta;              /* f32 [J,H], ACCUMULATED, or NULL */
} ts_kread_grad_args;

int ts_b200_kread_bwd(const ts_kread_args* args, const ts_kread_grad_args* grad, ts_stream_t stream);

/* ------------------------------------------------------------------ feature mass
 *
 * Query side of the feature-mass read (engine.dual_read_views.memory,
 * src/thetascan/_core/ops/engine.py:443-456): each temporal view divides the
 * query features by its own cumulative key-feature mass
 *   mass_t[f] = sum_{i<=t} w(t-i) phi_k[i][f]
 * (view.mass_cum: causal_prefix_sum, ema_cumsum or their stale difference,
 * src/thetascan/_core/ops/interface.py:58-107, 216-230, 278-279, 306-307)
 * before an unnormalized scan of that view:
 *   q_scaled = phi_q / (mass + eps)   (bf16, or f32 with q_scaled_f32)
 * w = 1 (log_alpha NULL), alpha_h^(t-i), or 1 - alpha_h^(t-i) (stale != 0).
 */
typedef struct ts_mass_args {
  int batch, heads, tokens, width;  /* width m: even, 2..512 */
  const void* phi_k;        /* bf16 [B,H,T,m] contiguous */
  const void* phi_q;        /* bf16 [B,H,T,m] contiguous */
  const float* log_alpha;   /* f32 [H] of the view, or NULL (plain prefix sum) */
  int stale;                /* the stale view's mass */
  float eps;
  void* q_scaled;           /* bf16 [B,H,T,m] out (forward) */
  const float* phi_q_f32;   /* f32 [B,H,T,m] phi(q), read instead of phi_q when set
                             * (ts_feature_args.phi_q_f32: one rounding, of the quotient) */
  int q_scaled_f32;         /* nonzero: q_scaled is f32 (8-byte aligned), unrounded, for a
                             * float32 scan; the backward's d mass then uses that quotient */
} ts_mass_args;

int ts_b200_mass_query_fwd(const ts_mass_args* args, ts_stream_t stream);

typedef struct ts_mass_grad_args {
  const void* dq_scaled;    /* [B,H,T,m] gradient of q_scaled */
  int dq_dtype;             /* TS_DTYPE_F32 or TS_DTYPE_BF16 */
  float* dphi_q;            /* f32 [B,H,T,m], ACCUMULATED into */
  float* dphi_k;            /* f32 [B,H,T,m], ACCUMULATED into (the mass path only) */
  float* dlog_alpha;        /* f32 [H], ACCUMULATED, or NULL */
  void* workspace;          /* ts_b200_mass_query_bwd_workspace_bytes(args) bytes */
  size_t workspace_bytes;
} ts_mass_grad_args;

size_t ts_b200_mass_query_bwd_workspace_bytes(const ts_mass_args* args);
int ts_b200_mass_query_bwd(const ts_mass_args* args, const ts_mass_grad_args* grad, ts_stream_t stream);

/* ------------------------------------------------------------------ GN rows
 *
 * Per-token row maps of the Gauss--Newton fast-weight family, forward and
 * backward: the write of engine._forward_theta0 / write_streams (one
 * Jacobian step, depth 1; src/thetascan/_core/ops/engine.py:161-340) and the
 * two read stages of engine.dual_read_views with the GN read normalisations
 * (engine.py:455-528).  The per-head linear maps between the stages
 * (W1 [H,m,d], W2 [H,d,m]: a = W1 k, O = W2 h, RS = (W2 o W2) s^2,
 * U = W2^T lam, ...) are plain GEMMs over all tokens of a head and run
 * outside these calls.  Every row tensor is f32 [B,H,T,width] contiguous
 * (width d, m, d+1, m+1 as given, or 1 for per-row scalars); d, m <= 256.
 *
 *   stage                in[]                                   out[]
 *   TS_GN_WRITE_PRE      a=W1 k [m], k [d]                      h [m], s2 [m], hh [1], kk [1]
 *        inv = (mean a^2 + eps)^-1/2, p = a inv - tau, h = sigma(p),
 *        s2 = (sigma'(p) inv)^2, hh = |h|^2, kk = |k|^2
 *   TS_GN_WRITE_LAM      v, k, O=W2 h, RS [d], hh, kk           lam [d]
 *        lam = (v - k - O) / (hh + kk RS + eps)
 *   TS_GN_WRITE_G        a [m], U=W2^T lam [m]                  g [m] = sigma'(p) U inv
 *   TS_GN_QUERY_PRE      a_q=W1 q [m]                           h0 [m] = relu2(a_q inv - tau)
 *   TS_GN_FEATURES       a_q [m], R [m(+1)] or NULL             hq [m] = sigma(pre inv - tau)
 *        pre = a_q + R[:m] / (R[m] + eps) (flags bit 0: R normalised by its
 *        mass column), a_q + R (bit 0 clear), a_q (R NULL)
 *   TS_GN_OUT            q, base=W2 hq [d], C [d(+1)]           y = q + base + C[:d] / (C[d] + eps)
 *        (flags bit 0; clear: y = q + base + C)
 *   TS_GN_OUT_BWD        dy [d], C [d+1]                        dC [d+1]
 *   TS_GN_FEATURES_BWD   a_q, R (as forward), dhq [m]           da_q [m], dR [m(+1)]
 *   TS_GN_QUERY_PRE_BWD  dh0 [m], a_q [m]                       da_q [m]
 *   TS_GN_WRITE_G_BWD    dg [m], a [m]                          du [m] = dg sigma'(p) inv
 *   TS_GN_WRITE_LAM_BWD  dlam, dlamW=W2 du, v, k, O, RS [d],    dv [d], drowsq [d], dk [d], dhh [1]
 *                        hh, kk
 *        dk holds the k terms outside a = W1 k (-dv + 2 k dkk)
 *   TS_GN_WRITE_PRE_BWD  dh [m], dhO=W2^T dv [m], ds2 [m],      da [m]
 *                        dhh [1], dg [m], U [m], a [m]
 * Backward stages add the threshold's gradient into dtau when both tau and
 * dtau are set; flags bit 1 makes FEATURES_BWD and QUERY_PRE_BWD add into
 * da_q instead of overwriting it.  tau is the relu2_threshold parameter
 * (its [H,m,1] tensor), subtracted after the normalisation.
 */
enum {
  TS_GN_RELU2 = 0,
  TS_GN_SILU = 1,
  TS_GN_TANH = 2
};

enum {
  TS_GN_WRITE_PRE = 1,
  TS_GN_WRITE_LAM = 2,
  TS_GN_WRITE_G = 3,
  TS_GN_QUERY_PRE = 4,
  TS_GN_FEATURES = 5,
  TS_GN_OUT = 6,
  TS_GN_OUT_BWD = 7,
  TS_GN_FEATURES_BWD = 8,
  TS_GN_QUERY_PRE_BWD = 9,
  TS_GN_WRITE_G_BWD = 10,
  TS_GN_WRITE_LAM_BWD = 11,
  TS_GN_WRITE_PRE_BWD = 12
};

typedef struct ts_gn_rows_args {
  int batch, heads, tokens;
  int d, m;                 /* head width, fast-net hidden width: 1..256 */
  int nonlinearity;         /* TS_GN_RELU2 / TS_GN_SILU / TS_GN_TANH (sigma of the net) */
  float eps;                /* the net's epsilon: normalisation, damping and read masses */
  const float* tau;         /* f32 [H,m] threshold, or NULL */
  float* dtau;              /* f32 [H,m], ACCUMULATED (backward stages), or NULL */
  int stage;                /* TS_GN_* */
  int flags;                /* bit 0: normalised read; bit 1: accumulate da_q */
  const float* in[8];       /* per stage, in the order of the table; 16-byte aligned not required */
  float* out[4];
  void* out_bf16;           /* forward stages: bf16 [B,H,T,width] copy of out[0] (the scans'
                             * operand), or NULL; with it out[0] may be NULL for WRITE_G and
                             * QUERY_PRE (g and h0 feed only the scans) */
} ts_gn_rows_args;

int ts_b200_gn_rows(const ts_gn_rows_args* args, ts_stream_t stream);

/* The GN mixer's q, k, v from its fused projection (block.py:577-599 of the
 * reference: the proj_qkv split, RoPE on q and k, then the L2 norm
 * x / max(|x|, eps)), and the backward of that map.  qkv is the projection
 * output f32 [B,T,3,H,d] contiguous; q, k, v f32 [B,H,T,d] contiguous.  RoPE
 * rotates adjacent channel pairs (2j, 2j+1) of the first `rot` channels
 * (even, 0 = none) by the phase tables cos/sin f32 [T, rot/2]. */
typedef struct ts_gn_prep_args {
  int batch, heads, tokens, d;   /* d <= 256 */
  int rot;
  const float* cos;
  const float* sin;
  float eps;
  const float* qkv;
  float* q;                      /* forward outputs */
  float* k;
  float* v;
  const float* dq;               /* backward inputs */
  const float* dk;
  const float* dv;
  float* dqkv;                   /* backward output, f32 [B,T,3,H,d] (written) */
} ts_gn_prep_args;

int ts_b200_gn_prep_fwd(const ts_gn_prep_args* args, ts_stream_t stream);
int ts_b200_gn_prep_bwd(const ts_gn_prep_args* args, ts_stream_t stream);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* THETASCAN_B200_H_ */
