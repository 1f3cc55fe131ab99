/*
 * thetascan_b200 -- C ABI of the B200 (sm_100a) ThetaScan hot path.
 *
 * The reference ThetaScan v0.1.0 is pure PyTorch and has no foreign-function
 * boundary; each entry point below names the reference interface it stands in
 * for (paths relative to the reference project root).  A Python host reaches
 * these through ctypes (thetascan_b200/_lib.py); any other host binds them the
 * same way.
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

/* ------------------------------------------------------------------ scan
 *
 * Multi-view inclusive causal scan, the contract of
 *   scan_chunk.linattn_views(q, k, v, retentions, chunk)
 *   (src/thetascan/_core/ops/scan_chunk.py:246-339)
 * out_r[t] = sum_{i<=t} w_r(t,i) (q_t . k_i) v_i  for every retention r, with
 * w = 1 (plain sum) or alpha_h^(t-i) (static per-head log-retention).  The
 * score tile q.k^T is formed once and shared by all retentions; the carried
 * state is f32.  Streams are bf16; their innermost dimension is contiguous.
 */
typedef struct ts_scan_args {
  int batch, heads, tokens;
  int dk;               /* key/query width, 1..256 */
  int dv;               /* payload width incl. the unit column if v_append_unit, 1..128 */
  const void* q;        /* bf16 [B,H,T,dk] */
  const void* k;        /* bf16 [B,H,T,dk] */
  const void* v;        /* bf16 [B,H,T,dv - v_append_unit] */
  int64_t q_strides[3]; /* element strides of batch, head, token */
  int64_t k_strides[3];
  int64_t v_strides[3];
  int v_append_unit;    /* 1: the payload is [v | 1] (key-mass read, engine.py:430) */
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
} ts_scan_args;

size_t ts_b200_scan_workspace_bytes(const ts_scan_args* args);

/* Forward of the multi-view scan (scan_chunk.py:246-339). */
int ts_b200_scan_fwd(const ts_scan_args* args, ts_stream_t stream);

/* Gradients of the multi-view scan (the autograd of scan_chunk.py:246-339,
 * pinned by tests/test_scan_chunk.py:271-340 of the reference).
 * dout[r]: bf16 [B,H,T,dv] contiguous.  dq/dk f32 or bf16 [B,H,T,dk], dv
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
} ts_scan_grad_args;

size_t ts_b200_scan_bwd_workspace_bytes(const ts_scan_args* fwd);
int ts_b200_scan_bwd(const ts_scan_args* fwd, const ts_scan_grad_args* grad, ts_stream_t stream);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* THETASCAN_B200_H_ */
