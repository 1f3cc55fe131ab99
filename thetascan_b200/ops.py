"""PyTorch custom operators over the C ABI (namespace ``thetascan_b200``).

Every GPU entry of the hot path that the mixer and the scan contract call is a
``torch.library`` custom op with a fake (meta) implementation and a
registered autograd formula, so that ``torch.compile`` traces a b200 mixer
into one graph (the reference pins single-graph tracing of every temporal
mode: tests/test_scan_chunk.py:663-738 of the reference project):

* ``thetascan_b200::scan_views_fwd`` / ``scan_views_bwd`` -- the multi-view
  scan of ``scan_chunk.linattn_views`` (src/thetascan/_core/ops/
  scan_chunk.py:246-339): the f32 reads of every retention (stacked) and the
  forward workspace that the backward reads;
* ``thetascan_b200::kernel_mixer_fwd`` / ``kernel_mixer_bwd`` -- the fused
  kernel-family core on post-RoPE/L2 ``q, k, v`` (the fused contract that
  replaces block.py:634-720): features, scan and key-mass read;
* ``thetascan_b200::kernel_mixer_qkv_fwd`` / ``kernel_mixer_qkv_bwd`` -- the
  same from the raw fused projection ``qkv [B,T,3Hd]``, with RoPE and the L2
  norm inside the feature kernels and the q/k/v gradients written into one
  ``d qkv``;
* ``thetascan_b200::gn_prep_fwd`` / ``gn_prep_bwd`` -- the GN mixer's q, k, v
  from its fused projection: RoPE and the L2 norm of q and k (block.py:
  577-599), one row kernel each way;
* ``thetascan_b200::gn_core_fwd`` / ``gn_core_bwd`` -- the Gauss--Newton
  family's core (write, two-stage read, bank combination; engine.py:161-340,
  455-528) on the GN row kernels, cuBLAS per-head maps and the scan kernels.

The forward ops return the intermediates their backward needs as extra
outputs (no state lives outside the graph).  Optional tensor inputs are
``None`` where the reference has no such parameter; gradients of those come
back as ``None``.  The ops run only on CUDA tensors and raise ``RuntimeError``
otherwise; they never fall back to a CPU implementation.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch
from torch import Tensor

from . import _lib

LIB = "thetascan_b200"


def _require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("b200 backend requires CUDA tensors")


# --------------------------------------------------------------------------- workspace sizes

def _scan_workspace_nbytes(B, H, T, dk, dv_payload, n_unit, present, stale, f32_streams, backward=False,
                           streams=None):
    """Workspace bytes of a scan call of this shape (the C ABI's size query,
    answered from shapes alone with placeholder pointers; nothing is read)."""
    lib = _lib.load()
    a = _lib.ScanArgs()
    a.batch, a.heads, a.tokens, a.dk = B, H, T, dk
    a.dv = dv_payload + n_unit
    a.q = a.k = a.v = 256
    a.q_strides = a.k_strides = _lib.c_int64_3(H * T * dk, T * dk, dk)
    a.v_strides = _lib.c_int64_3(H * T * dv_payload, T * dv_payload, dv_payload)
    a.v_append_unit = n_unit
    a.n_retentions = len(present)
    for i, p in enumerate(present):
        stream = bool(streams and streams[i])
        a.log_alpha[i] = 256 if (p and not stream) else None
        a.log_alpha_stream[i] = 256 if (p and stream) else None
        a.stale[i] = 1 if (stale and stale[i]) else 0
        a.out[i] = 256
    a.out_dtype = _lib.TS_DTYPE_F32
    a.f32_streams = 1 if f32_streams else 0
    fn = lib.ts_b200_scan_bwd_workspace_bytes if backward else lib.ts_b200_scan_workspace_bytes
    nbytes = fn(ctypes.byref(a))
    if nbytes == 0:
        _lib.check(_lib.last_error()[0] or _lib.TS_ERR_VALUE)
    return int(nbytes)


# --------------------------------------------------------------------------- scan contract

@torch.library.custom_op(f"{LIB}::scan_views_fwd", mutates_args=())
def scan_views_fwd(q: Tensor, k: Tensor, v: Tensor, log_alphas: list[Tensor], present: list[bool],
                   append_unit: int, stale: list[bool], round_streams: bool) -> tuple[Tensor, Tensor]:
    """Reads f32 ``[R,B,H,T,Dv(+unit)]`` of every retention and the forward
    workspace.  Retention r is the plain sum where ``present[r]`` is False,
    else the next tensor of ``log_alphas`` (static ``[H]``, or a per-token
    stream ``[B,H,T,1]``, which runs the float32 CUDA-core kernels).
    ``round_streams``: float32 q/k/v are rounded to bf16 and run on the
    tensor cores (the GN family's per-token math is float32)."""
    from .scan import _scan_fwd_impl
    _require_cuda(q, k, v, *log_alphas)
    return _scan_fwd_impl(q, k, v, _retentions(log_alphas, present), append_unit, stale, round_streams)


def _retentions(log_alphas, present):
    it = iter(log_alphas)
    return [next(it) if p else None for p in present]


def _stream_flags(log_alphas, present):
    return [r is not None and r.ndim == 4 for r in _retentions(log_alphas, present)]


@scan_views_fwd.register_fake
def _(q, k, v, log_alphas, present, append_unit, stale, round_streams):
    B, H, T, dk = (int(s) for s in q.shape)
    dvp = int(v.shape[-1])
    streams = _stream_flags(log_alphas, present)
    f32 = any(streams) or (q.dtype == torch.float32 and not round_streams)
    outs = q.new_empty(len(present), B, H, T, dvp + append_unit, dtype=torch.float32)
    nbytes = _scan_workspace_nbytes(B, H, T, dk, dvp, append_unit, list(present), stale, f32, streams=streams)
    return outs, q.new_empty(nbytes, dtype=torch.uint8)


@torch.library.custom_op(f"{LIB}::scan_views_bwd", mutates_args=())
def scan_views_bwd(douts: Tensor, q: Tensor, k: Tensor, v: Tensor, log_alphas: list[Tensor], present: list[bool],
                   outs: Tensor, ws: Tensor, append_unit: int, stale: list[bool],
                   round_streams: bool) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor]:
    """Gradients of q, k, v (f32, v without the unit columns), of every static
    retention (f32 ``[R,H]``, zero rows for the plain sum and for streams) and
    of the S per-token retention streams (f32 ``[S,B,H,T]``, in order)."""
    from .scan import _scan_bwd_impl
    _require_cuda(douts, q, k, v, outs, ws, *log_alphas)
    return _scan_bwd_impl(douts, q, k, v, _retentions(log_alphas, present), outs, ws, append_unit, stale,
                          round_streams)


@scan_views_bwd.register_fake
def _(douts, q, k, v, log_alphas, present, outs, ws, append_unit, stale, round_streams):
    f = torch.float32
    n_streams = sum(_stream_flags(log_alphas, present))
    return (q.new_empty(q.shape, dtype=f), k.new_empty(k.shape, dtype=f), v.new_empty(v.shape, dtype=f),
            q.new_empty(len(present), q.shape[1], dtype=f), q.new_empty(n_streams, *q.shape[:3], dtype=f))


def _scan_setup(ctx, inputs, output):
    q, k, v, log_alphas, present, append_unit, stale, round_streams = inputs
    outs, ws = output
    ctx.present = list(present)
    ctx.ret_meta = [(r.dtype, r.shape) for r in log_alphas]
    ctx.args = (append_unit, list(stale), round_streams)
    ctx.dtypes = (q.dtype, k.dtype, v.dtype)
    ctx.mark_non_differentiable(ws)
    ctx.set_materialize_grads(False)
    ctx.save_for_backward(q, k, v, outs, ws, *log_alphas)


def _scan_backward(ctx, douts, dws):
    q, k, v, outs, ws, *log_alphas = ctx.saved_tensors
    append_unit, stale, round_streams = ctx.args
    if douts is None:
        douts = torch.zeros_like(outs)
    dq, dk, dv, dla, dstream = scan_views_bwd(douts, q, k, v, log_alphas, ctx.present, outs, ws, append_unit,
                                              stale, round_streams)
    qd, kd, vd = ctx.dtypes
    rows = [i for i, p in enumerate(ctx.present) if p]
    dret, s_index = [], 0
    for i, (dtype, shape) in zip(rows, ctx.ret_meta):
        if len(shape) == 4:
            dret.append(dstream[s_index].to(dtype).reshape(shape))
            s_index += 1
        else:
            dret.append(dla[i].to(dtype).reshape(shape))
    return dq.to(qd), dk.to(kd), dv.to(vd), dret, None, None, None, None


torch.library.register_autograd(f"{LIB}::scan_views_fwd", _scan_backward, setup_context=_scan_setup)


# --------------------------------------------------------------------------- fused kernel-family core

def _spec(kind, mode, eps, gain, basis, bound, spline_scale, sparsity="none", temperature=0.25):
    from .kernel import KernelSpec
    return KernelSpec(kind=kind, mode=mode, eps=eps, gain=gain, basis=basis, bound=bound,
                      spline_scale=spline_scale, read="key_mass", sparsity=sparsity, temperature=temperature)


def _fake_core_outputs(like, B, H, T, d, W1, kind, basis, log_alphas, mode):
    from .kernel import MASS_COLS
    m = int(W1.shape[1]) * (basis if kind == "projected_bspline" else 1)
    n = 1 + (0 if log_alphas is None else int(log_alphas.shape[0]))
    bf, f = torch.bfloat16, torch.float32
    stale = [False] + [mode == "stale"] * (n - 1)
    nbytes = _scan_workspace_nbytes(B, H, T, m, d, MASS_COLS, [False] + [True] * (n - 1), stale, False)
    return (like.new_empty(B, T, H, d, dtype=bf), like.new_empty(B, H, T, m, dtype=bf),
            like.new_empty(B, H, T, m, dtype=bf), like.new_empty(B, H, T, d, dtype=f),
            like.new_empty(n, B, H, T, d + MASS_COLS, dtype=f), like.new_empty(nbytes, dtype=torch.uint8))


def _grad_or_empty(g, like, ref):
    """The gradient in its input's dtype, or an empty tensor for an absent input."""
    return ref.new_empty(0) if like is None else g.to(like.dtype)


def _control_grads(g, controls, ref):
    """Gradients of the six feature controls (threshold, score bias, gain,
    spline scale, relative threshold, sparse blend), empty where absent."""
    keys = ("thr", "bias", "gain", "scale", "rho", "alpha")
    return [_grad_or_empty(g[key], c, ref) for key, c in zip(keys, controls)]


# Tensor inputs of the fused core ops after the streams and weights: the six
# feature controls (threshold, score_bias, gain, spline_scale,
# relative_threshold, sparse_blend), then log_alphas and etas.
_N_CORE_TENSORS = 13


@torch.library.custom_op(f"{LIB}::kernel_mixer_fwd", mutates_args=())
def kernel_mixer_fwd(q: Tensor, k: Tensor, v: Tensor, W1: Tensor, W2: Tensor, threshold: Optional[Tensor],
                     score_bias: Optional[Tensor], gain: Optional[Tensor], spline_scale: Optional[Tensor],
                     relative_threshold: Optional[Tensor], sparse_blend: Optional[Tensor],
                     log_alphas: Optional[Tensor], etas: Optional[Tensor], kind: str, mode: str, eps: float,
                     gain_scalar: float, basis: int, bound: float, spline_scale_scalar: float, sparsity: str,
                     temperature: float) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor, Tensor]:
    """``y [B,T,H,d]`` bf16 plus (phi_q, phi_k, y0, stacked reads, workspace)."""
    from .kernel import _controls, _core_forward
    _require_cuda(q, k, v, W1, W2, threshold, score_bias, gain, spline_scale, relative_threshold, sparse_blend,
                  log_alphas, etas)
    spec = _spec(kind, mode, eps, gain_scalar, basis, bound, spline_scale_scalar, sparsity, temperature)
    ctl = _controls(threshold, score_bias, gain, spline_scale, relative_threshold, sparse_blend)
    y, st = _core_forward(spec, q, k, v, W1, W2, ctl, log_alphas, etas, None)
    return y, st["phi_q"], st["phi_k"], st["y0"], st["slots_all"], st["ws"]


@kernel_mixer_fwd.register_fake
def _(q, k, v, W1, W2, threshold, score_bias, gain, spline_scale, relative_threshold, sparse_blend, log_alphas,
      etas, kind, mode, eps, gain_scalar, basis, bound, spline_scale_scalar, sparsity, temperature):
    B, H, T, d = (int(s) for s in q.shape)
    return _fake_core_outputs(q, B, H, T, d, W1, kind, basis, log_alphas, mode)


@torch.library.custom_op(f"{LIB}::kernel_mixer_bwd", mutates_args=())
def kernel_mixer_bwd(dy: Tensor, q: Tensor, k: Tensor, v: Tensor, W1: Tensor, W2: Tensor,
                     threshold: Optional[Tensor], score_bias: Optional[Tensor], gain: Optional[Tensor],
                     spline_scale: Optional[Tensor], relative_threshold: Optional[Tensor],
                     sparse_blend: Optional[Tensor], log_alphas: Optional[Tensor], etas: Optional[Tensor],
                     phi_q: Tensor, phi_k: Tensor, y0: Tensor, slots: Tensor, ws: Tensor, kind: str, mode: str,
                     eps: float, gain_scalar: float, basis: int, bound: float, spline_scale_scalar: float,
                     sparsity: str, temperature: float) -> list[Tensor]:
    """Gradients of q, k, v, W1, W2, the six controls, log_alphas and etas
    (an empty tensor where the input is None)."""
    from .kernel import _controls, _core_backward, _saved_state
    _require_cuda(dy, q, k, v, W1, W2, phi_q, phi_k, y0, slots, ws)
    spec = _spec(kind, mode, eps, gain_scalar, basis, bound, spline_scale_scalar, sparsity, temperature)
    controls = (threshold, score_bias, gain, spline_scale, relative_threshold, sparse_blend)
    ctl = _controls(*controls)
    st = _saved_state(W1, W2, log_alphas, etas, phi_q, phi_k, y0, slots, ws)
    g = _core_backward(spec, q, k, v, st, ctl, dy, None, None, None, None)
    d = q.shape[-1]
    return [g["dq"].to(q.dtype), g["dk"].to(k.dtype), g["dvaug"][..., :d].to(v.dtype).contiguous(),
            g["dW1"].to(W1.dtype), g["dW2"].to(W2.dtype).contiguous(), *_control_grads(g, controls, q),
            _grad_or_empty(g["dla"], log_alphas, q), _grad_or_empty(g["deta"], etas, q)]


@kernel_mixer_bwd.register_fake
def _(dy, q, k, v, W1, W2, threshold, score_bias, gain, spline_scale, relative_threshold, sparse_blend, log_alphas,
      etas, phi_q, phi_k, y0, slots, ws, kind, mode, eps, gain_scalar, basis, bound, spline_scale_scalar, sparsity,
      temperature):
    def like(t, ref):
        return ref.new_empty(0) if t is None else torch.empty_like(t)
    return [torch.empty_like(q), torch.empty_like(k), torch.empty_like(v), torch.empty_like(W1),
            torch.empty_like(W2), *[like(c, q) for c in (threshold, score_bias, gain, spline_scale,
                                                         relative_threshold, sparse_blend)],
            like(log_alphas, q), like(etas, q)]


def _none_if_absent(grads, inputs):
    return [None if x is None else g for g, x in zip(grads, inputs)]


def _core_setup(ctx, inputs, output):
    tensors, scalars = inputs[:_N_CORE_TENSORS], inputs[_N_CORE_TENSORS:]
    _, phi_q, phi_k, y0, slots, ws = output
    ctx.mark_non_differentiable(phi_q, phi_k, y0, slots, ws)
    # the saved intermediates take no gradient: do not fill zeros for them
    ctx.set_materialize_grads(False)
    ctx.scalars = scalars
    ctx.present = [t is not None for t in tensors]
    ctx.save_for_backward(*[t for t in tensors if t is not None], phi_q, phi_k, y0, slots, ws)


def _unpack_saved(ctx, n_inputs):
    saved = list(ctx.saved_tensors)
    inputs = []
    for p in ctx.present[:n_inputs]:
        inputs.append(saved.pop(0) if p else None)
    return inputs, saved


def _core_backward_op(ctx, dy, *unused):
    inputs, (phi_q, phi_k, y0, slots, ws) = _unpack_saved(ctx, _N_CORE_TENSORS)
    grads = kernel_mixer_bwd(dy, *inputs, phi_q, phi_k, y0, slots, ws, *ctx.scalars)
    return (*_none_if_absent(grads, inputs), *([None] * len(ctx.scalars)))


torch.library.register_autograd(f"{LIB}::kernel_mixer_fwd", _core_backward_op, setup_context=_core_setup)


@torch.library.custom_op(f"{LIB}::kernel_mixer_qkv_fwd", mutates_args=())
def kernel_mixer_qkv_fwd(qkv: Tensor, W1: Tensor, W2: Tensor, threshold: Optional[Tensor],
                         score_bias: Optional[Tensor], gain: Optional[Tensor], spline_scale: Optional[Tensor],
                         relative_threshold: Optional[Tensor], sparse_blend: Optional[Tensor],
                         log_alphas: Optional[Tensor], etas: Optional[Tensor], rope_cos: Optional[Tensor],
                         rope_sin: Optional[Tensor], heads: int, rope_rot: int, l2norm_eps: float, kind: str,
                         mode: str, eps: float, gain_scalar: float, basis: int, bound: float,
                         spline_scale_scalar: float, sparsity: str,
                         temperature: float) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor, Tensor]:
    """The fused core from the raw projection ``qkv [B,T,3Hd]`` (RoPE and L2
    norm inside the feature kernels)."""
    from .kernel import Prologue, _controls, _core_forward, _qkv_views
    _require_cuda(qkv, W1, W2, threshold, score_bias, gain, spline_scale, relative_threshold, sparse_blend,
                  log_alphas, etas, rope_cos, rope_sin)
    spec = _spec(kind, mode, eps, gain_scalar, basis, bound, spline_scale_scalar, sparsity, temperature)
    d = qkv.shape[-1] // (3 * heads)
    q, k, v = _qkv_views(qkv, heads, d)
    ctl = _controls(threshold, score_bias, gain, spline_scale, relative_threshold, sparse_blend)
    prologue = Prologue(rope_rot, rope_cos, rope_sin, None if l2norm_eps < 0 else l2norm_eps)
    y, st = _core_forward(spec, q, k, v, W1, W2, ctl, log_alphas, etas, prologue)
    return y, st["phi_q"], st["phi_k"], st["y0"], st["slots_all"], st["ws"]


@kernel_mixer_qkv_fwd.register_fake
def _(qkv, W1, W2, threshold, score_bias, gain, spline_scale, relative_threshold, sparse_blend, log_alphas, etas,
      rope_cos, rope_sin, heads, rope_rot, l2norm_eps, kind, mode, eps, gain_scalar, basis, bound,
      spline_scale_scalar, sparsity, temperature):
    B, T, width = (int(s) for s in qkv.shape)
    d = width // (3 * heads)
    return _fake_core_outputs(qkv, B, heads, T, d, W1, kind, basis, log_alphas, mode)


@torch.library.custom_op(f"{LIB}::kernel_mixer_qkv_bwd", mutates_args=())
def kernel_mixer_qkv_bwd(dy: Tensor, qkv: Tensor, W1: Tensor, W2: Tensor, threshold: Optional[Tensor],
                         score_bias: Optional[Tensor], gain: Optional[Tensor], spline_scale: Optional[Tensor],
                         relative_threshold: Optional[Tensor], sparse_blend: Optional[Tensor],
                         log_alphas: Optional[Tensor], etas: Optional[Tensor], rope_cos: Optional[Tensor],
                         rope_sin: Optional[Tensor], phi_q: Tensor, phi_k: Tensor, y0: Tensor, slots: Tensor,
                         ws: Tensor, heads: int, rope_rot: int, l2norm_eps: float, kind: str, mode: str, eps: float,
                         gain_scalar: float, basis: int, bound: float, spline_scale_scalar: float, sparsity: str,
                         temperature: float) -> list[Tensor]:
    """Gradients of qkv, W1, W2, the six controls, log_alphas and etas."""
    from .kernel import Prologue, _controls, _core_backward, _qkv_views, _saved_state
    _require_cuda(dy, qkv, W1, W2, phi_q, phi_k, y0, slots, ws)
    spec = _spec(kind, mode, eps, gain_scalar, basis, bound, spline_scale_scalar, sparsity, temperature)
    d = qkv.shape[-1] // (3 * heads)
    q, k, v = _qkv_views(qkv, heads, d)
    dqkv = torch.empty_like(qkv)
    dq, dk, dv = _qkv_views(dqkv, heads, d)
    controls = (threshold, score_bias, gain, spline_scale, relative_threshold, sparse_blend)
    ctl = _controls(*controls)
    st = _saved_state(W1, W2, log_alphas, etas, phi_q, phi_k, y0, slots, ws)
    prologue = Prologue(rope_rot, rope_cos, rope_sin, None if l2norm_eps < 0 else l2norm_eps)
    g = _core_backward(spec, q, k, v, st, ctl, dy, prologue, dq, dk, dv)
    return [dqkv, g["dW1"].to(W1.dtype), g["dW2"].to(W2.dtype).contiguous(), *_control_grads(g, controls, qkv),
            _grad_or_empty(g["dla"], log_alphas, qkv), _grad_or_empty(g["deta"], etas, qkv)]


@kernel_mixer_qkv_bwd.register_fake
def _(dy, qkv, W1, W2, threshold, score_bias, gain, spline_scale, relative_threshold, sparse_blend, log_alphas, etas,
      rope_cos, rope_sin, phi_q, phi_k, y0, slots, ws, heads, rope_rot, l2norm_eps, kind, mode, eps, gain_scalar,
      basis, bound, spline_scale_scalar, sparsity, temperature):
    def like(t):
        return qkv.new_empty(0) if t is None else torch.empty_like(t)
    return [torch.empty_like(qkv), torch.empty_like(W1), torch.empty_like(W2),
            *[like(c) for c in (threshold, score_bias, gain, spline_scale, relative_threshold, sparse_blend)],
            like(log_alphas), like(etas)]


def _qkv_setup(ctx, inputs, output):
    tensors, scalars = inputs[:_N_CORE_TENSORS], inputs[_N_CORE_TENSORS:]
    _, phi_q, phi_k, y0, slots, ws = output
    ctx.mark_non_differentiable(phi_q, phi_k, y0, slots, ws)
    # the saved intermediates take no gradient: do not fill zeros for them
    ctx.set_materialize_grads(False)
    ctx.scalars = scalars
    ctx.present = [t is not None for t in tensors]
    ctx.save_for_backward(*[t for t in tensors if t is not None], phi_q, phi_k, y0, slots, ws)


def _qkv_backward_op(ctx, dy, *unused):
    inputs, (phi_q, phi_k, y0, slots, ws) = _unpack_saved(ctx, _N_CORE_TENSORS)
    grads = kernel_mixer_qkv_bwd(dy, *inputs, phi_q, phi_k, y0, slots, ws, *ctx.scalars)
    # qkv, W1, W2, 6 controls, log_alphas, etas; the rope tables take no gradient
    return (*_none_if_absent(grads, inputs[:11]), None, None, *([None] * len(ctx.scalars)))


torch.library.register_autograd(f"{LIB}::kernel_mixer_qkv_fwd", _qkv_backward_op, setup_context=_qkv_setup)


# --------------------------------------------------------------------------- streaming scan

@torch.library.custom_op(f"{LIB}::scan_views_stream_fwd", mutates_args=())
def scan_views_stream_fwd(q: Tensor, k: Tensor, v: Tensor, log_alphas: list[Tensor], present: list[bool],
                          append_unit: int, state: Optional[Tensor]) -> tuple[Tensor, Tensor, Tensor]:
    """One segment of a streamed scan: f32 reads ``[R,B,H,T,Dv(+unit)]``
    continuing from ``state`` (f32 ``[B,H,R,Dk,Dv]``, None = zero), the state
    after the segment, and the forward workspace."""
    from .scan import _stream_fwd_impl
    _require_cuda(q, k, v, state, *log_alphas)
    return _stream_fwd_impl(q, k, v, _retentions(log_alphas, present), append_unit, state)


@scan_views_stream_fwd.register_fake
def _(q, k, v, log_alphas, present, append_unit, state):
    B, H, T, dk = (int(s) for s in q.shape)
    dvp = int(v.shape[-1])
    R = len(present)
    outs = q.new_empty(R, B, H, T, dvp + append_unit, dtype=torch.float32)
    new_state = q.new_empty(B, H, R, dk, dvp + append_unit, dtype=torch.float32)
    nbytes = _scan_workspace_nbytes(B, H, T, dk, dvp, append_unit, list(present), [False] * R, False)
    return outs, new_state, q.new_empty(nbytes, dtype=torch.uint8)


@torch.library.custom_op(f"{LIB}::scan_views_stream_bwd", mutates_args=())
def scan_views_stream_bwd(douts: Tensor, dstate: Tensor, q: Tensor, k: Tensor, v: Tensor, log_alphas: list[Tensor],
                          present: list[bool], outs: Tensor, ws: Tensor, append_unit: int,
                          state: Optional[Tensor]) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor]:
    """Gradients of q, k, v, every retention (``[R,H]``) and of the entering
    state (empty when there was none) from those of the reads and the
    leaving state."""
    from .scan import _stream_bwd_impl
    _require_cuda(douts, dstate, q, k, v, outs, ws, state, *log_alphas)
    return _stream_bwd_impl(douts, dstate, q, k, v, _retentions(log_alphas, present), outs, ws, append_unit, state)


@scan_views_stream_bwd.register_fake
def _(douts, dstate, q, k, v, log_alphas, present, outs, ws, append_unit, state):
    f = torch.float32
    return (q.new_empty(q.shape, dtype=f), k.new_empty(k.shape, dtype=f), v.new_empty(v.shape, dtype=f),
            q.new_empty(len(present), q.shape[1], dtype=f),
            q.new_empty(0) if state is None else torch.empty_like(state))


def _stream_setup(ctx, inputs, output):
    q, k, v, log_alphas, present, append_unit, state = inputs
    outs, new_state, ws = output
    ctx.present = list(present)
    ctx.ret_meta = [(r.dtype, r.shape) for r in log_alphas]
    ctx.append_unit = append_unit
    ctx.has_state = state is not None
    ctx.dtypes = (q.dtype, k.dtype, v.dtype)
    ctx.mark_non_differentiable(ws)
    ctx.set_materialize_grads(False)
    ctx.save_for_backward(q, k, v, outs, new_state, ws, state, *log_alphas)


def _stream_backward(ctx, douts, dstate, dws):
    q, k, v, outs, new_state, ws, state, *log_alphas = ctx.saved_tensors
    if douts is None:
        douts = torch.zeros_like(outs)
    if dstate is None:
        dstate = torch.zeros_like(new_state)
    dq, dk, dv, dla, dinit = scan_views_stream_bwd(douts, dstate, q, k, v, log_alphas, ctx.present, outs, ws,
                                                   ctx.append_unit, state)
    qd, kd, vd = ctx.dtypes
    rows = [i for i, p in enumerate(ctx.present) if p]
    dret = [dla[i].to(meta[0]).reshape(meta[1]) for i, meta in zip(rows, ctx.ret_meta)]
    return (dq.to(qd), dk.to(kd), dv.to(vd), dret, None, None, dinit if ctx.has_state else None)


torch.library.register_autograd(f"{LIB}::scan_views_stream_fwd", _stream_backward, setup_context=_stream_setup)


# --------------------------------------------------------------------------- GN core

@torch.library.custom_op(f"{LIB}::gn_core_fwd", mutates_args=())
def gn_core_fwd(q: Tensor, k: Tensor, v: Tensor, W1: Tensor, W2: Tensor, tau: Optional[Tensor],
                log_alphas: Optional[Tensor], etas: Optional[Tensor], nonlin: str, read_norm: bool,
                read_norm_w1: bool, mode: str, eps: float, steps: int) -> tuple[Tensor, list[Tensor]]:
    """GN core ``y [B,H,T,d]`` f32 from f32 post-RoPE/L2 ``q, k, v`` plus the
    intermediates of its backward (write streams, stage reads, scan states)."""
    from .gn import _gn_forward
    _require_cuda(q, k, v, W1, W2, tau, log_alphas, etas)
    return _gn_forward(q, k, v, W1, W2, tau, log_alphas, etas, nonlin, read_norm, read_norm_w1, mode, eps, False,
                       steps)


@gn_core_fwd.register_fake
def _(q, k, v, W1, W2, tau, log_alphas, etas, nonlin, read_norm, read_norm_w1, mode, eps, steps):
    from .gn import _gn_forward
    return _gn_forward(q, k, v, W1, W2, tau, log_alphas, etas, nonlin, read_norm, read_norm_w1, mode, eps, True,
                       steps)


@torch.library.custom_op(f"{LIB}::gn_core_bwd", mutates_args=())
def gn_core_bwd(dy: Tensor, q: Tensor, k: Tensor, v: Tensor, W1: Tensor, W2: Tensor, tau: Optional[Tensor],
                log_alphas: Optional[Tensor], etas: Optional[Tensor], saved: list[Tensor], nonlin: str,
                read_norm: bool, read_norm_w1: bool, mode: str, eps: float,
                steps: int) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor]:
    """Gradients of q, k, v, W1, W2 (f32) and of tau ``[H,m]``, the bank's
    log-retentions and etas ``[J,H]`` (empty where the input is absent)."""
    from .gn import _gn_backward
    _require_cuda(dy, q, k, v, W1, W2, tau, log_alphas, etas)
    return _gn_outputs(_gn_backward(dy, q, k, v, W1, W2, tau, log_alphas, etas, list(saved), nonlin, read_norm,
                                    read_norm_w1, mode, eps, False, steps), q)


def _gn_outputs(grads, q):
    return tuple(q.new_empty(0) if g_ is None else g_.contiguous() for g_ in grads)


@gn_core_bwd.register_fake
def _(dy, q, k, v, W1, W2, tau, log_alphas, etas, saved, nonlin, read_norm, read_norm_w1, mode, eps, steps):
    from .gn import _gn_backward
    return _gn_outputs(_gn_backward(dy, q, k, v, W1, W2, tau, log_alphas, etas, list(saved), nonlin, read_norm,
                                    read_norm_w1, mode, eps, True, steps), q)


def _gn_setup(ctx, inputs, output):
    q, k, v, W1, W2, tau, log_alphas, etas, nonlin, read_norm, read_norm_w1, mode, eps, steps = inputs
    y, saved = output
    ctx.args = (nonlin, read_norm, read_norm_w1, mode, eps, steps)
    ctx.present = (tau is not None, log_alphas is not None, etas is not None)
    ctx.meta = [(t.dtype, t.shape) if t is not None else None for t in (q, k, v, W1, W2, tau, log_alphas, etas)]
    ctx.n_saved = len(saved)
    ctx.mark_non_differentiable(*saved)
    ctx.set_materialize_grads(False)
    ctx.save_for_backward(q, k, v, W1, W2, *[t for t in (tau, log_alphas, etas) if t is not None], *saved)


def _gn_backward_fn(ctx, dy, dsaved):
    t = list(ctx.saved_tensors)
    q, k, v, W1, W2 = t[:5]
    rest = t[5:]
    opt = []
    for p in ctx.present:
        opt.append(rest.pop(0) if p else None)
    tau, log_alphas, etas = opt
    if dy is None:
        dy = torch.zeros_like(q, dtype=torch.float32)
    grads = gn_core_bwd(dy, q, k, v, W1, W2, tau, log_alphas, etas, rest, *ctx.args)
    out = []
    for g_, meta in zip(grads, ctx.meta):
        out.append(None if meta is None else g_.to(meta[0]).reshape(meta[1]))
    return (*out, None, None, None, None, None, None)


torch.library.register_autograd(f"{LIB}::gn_core_fwd", _gn_backward_fn, setup_context=_gn_setup)


# --------------------------------------------------------------------------- GN stream preparation

def _gn_prep_call(fn, qkv, cos, sin, rot, heads, eps, outs=None, grads=None):
    B, T, w = (int(x) for x in qkv.shape)
    d = w // (3 * heads)
    a = _lib.GnPrepArgs()
    a.batch, a.heads, a.tokens, a.d, a.rot, a.eps = B, heads, T, d, rot, eps
    a.cos, a.sin = (cos.data_ptr(), sin.data_ptr()) if rot else (None, None)
    a.qkv = qkv.data_ptr()
    if outs is not None:
        a.q, a.k, a.v = (x.data_ptr() for x in outs)
    if grads is not None:
        (a.dq, a.dk, a.dv), a.dqkv = (x.data_ptr() for x in grads[:3]), grads[3].data_ptr()
    _lib.check(fn(ctypes.byref(a), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))


@torch.library.custom_op(f"{LIB}::gn_prep_fwd", mutates_args=())
def gn_prep_fwd(qkv: Tensor, cos: Tensor, sin: Tensor, rot: int, heads: int,
                eps: float) -> tuple[Tensor, Tensor, Tensor]:
    """q, k, v f32 ``[B,H,T,d]`` from the f32 fused projection ``[B,T,3Hd]``:
    RoPE on the first ``rot`` channels (phase tables ``[T, rot/2]``) and the
    L2 norm of q and k."""
    _require_cuda(qkv, cos, sin)
    qkv = qkv.contiguous()
    B, T, w = qkv.shape
    d = w // (3 * heads)
    outs = [qkv.new_empty(B, heads, T, d) for _ in range(3)]
    _gn_prep_call(_lib.load().ts_b200_gn_prep_fwd, qkv, cos.contiguous(), sin.contiguous(), rot, heads, eps,
                  outs=outs)
    return tuple(outs)


@gn_prep_fwd.register_fake
def _(qkv, cos, sin, rot, heads, eps):
    B, T, w = qkv.shape
    d = w // (3 * heads)
    return tuple(qkv.new_empty(B, heads, T, d) for _ in range(3))


@torch.library.custom_op(f"{LIB}::gn_prep_bwd", mutates_args=())
def gn_prep_bwd(dq: Tensor, dk: Tensor, dv: Tensor, qkv: Tensor, cos: Tensor, sin: Tensor, rot: int, heads: int,
                eps: float) -> Tensor:
    """Gradient of the fused projection ``[B,T,3Hd]`` (f32)."""
    _require_cuda(dq, dk, dv, qkv, cos, sin)
    qkv = qkv.contiguous()
    dqkv = torch.empty_like(qkv)
    grads = [g_.float().contiguous() for g_ in (dq, dk, dv)] + [dqkv]
    _gn_prep_call(_lib.load().ts_b200_gn_prep_bwd, qkv, cos.contiguous(), sin.contiguous(), rot, heads, eps,
                  grads=grads)
    return dqkv


@gn_prep_bwd.register_fake
def _(dq, dk, dv, qkv, cos, sin, rot, heads, eps):
    return torch.empty_like(qkv)


def _gn_prep_setup(ctx, inputs, output):
    qkv, cos, sin, rot, heads, eps = inputs
    ctx.args = (rot, heads, eps)
    ctx.save_for_backward(qkv, cos, sin)


def _gn_prep_backward(ctx, dq, dk, dv):
    qkv, cos, sin = ctx.saved_tensors
    z = None
    grads = [g_ if g_ is not None else torch.zeros(qkv.shape[0], ctx.args[1], qkv.shape[1],
                                                   qkv.shape[2] // (3 * ctx.args[1]), device=qkv.device)
             for g_ in (dq, dk, dv)]
    return gn_prep_bwd(*grads, qkv, cos, sin, *ctx.args), z, z, None, None, None


torch.library.register_autograd(f"{LIB}::gn_prep_fwd", _gn_prep_backward, setup_context=_gn_prep_setup)
