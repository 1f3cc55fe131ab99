"""Fused kernel-family hot path: write features, multi-view scan, normalized read.

``kernel_core`` is the B200 counterpart of the reference chain
``engine.write_streams`` + ``engine.dual_read`` per temporal view +
``read_with_temporal`` blending (src/thetascan/_core/ops/engine.py:260-553,
src/thetascan/_core/modules/block.py:644-718) for the kernel family with a
key-mass normalized read.  Forward, all on the GPU through the C ABI:

1. ``ts_b200_feature_fwd``: phi(k), phi(q) and y0 = q + W2 phi(q)
2. ``ts_b200_scan_fwd``: the augmented reads [N | D] of every retention slot
   (plain sum, then one per recency branch), sharing each score tile
3. ``ts_b200_kread_fwd``: y = y0 + blended N / (D + eps), token-major

and the backward runs the three in reverse.  Inputs are bf16 streams; the
effective weights and controls are cast to what the kernels read.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib
from .scan import _build_args, _stream, _workspace

# Mass columns of every scan read [N | D | D]: the read backward hands the
# mass gradient to the scan as bf16 hi + lo (see ts_kread_args.mass_columns).
MASS_COLS = 2

KINDS = {"relu2_ridge": _lib.TS_FEATURE_RELU2, "softmax_partition": _lib.TS_FEATURE_SOFTMAX,
         "projected_bspline": _lib.TS_FEATURE_BSPLINE}
MODES = {"sum": _lib.TS_VIEWS_SUM, "fast": _lib.TS_VIEWS_FAST, "stale": _lib.TS_VIEWS_STALE}


@dataclass(frozen=True)
class KernelSpec:
    """Static description of the feature map and views of one mixer."""

    kind: str                   # relu2_ridge | softmax_partition | projected_bspline
    mode: str = "sum"           # sum | fast | stale
    eps: float = 1e-6
    gain: float = 8.0           # fixed softmax sharpness when no learned gain
    basis: int = 8              # B-spline basis per projection
    bound: float = 3.0
    spline_scale: float = 1.0   # fixed B-spline scale when no learned scale
    read: str = "key_mass"      # key_mass | feature_mass | none (engine.py:402-456)
    sparsity: str = "none"      # none | relative_soft | relative_st | relative_st_blend (softmax partition)
    temperature: float = 0.25   # relative-threshold gate temperature


SPARSITY = {"none": 0, "relative_soft": 1, "relative_st": 2, "relative_st_blend": 3}


def _ptr(t):
    return None if t is None else t.data_ptr()


def _f32(t):
    return None if t is None else t.detach().to(torch.float32).contiguous()


def _feature_args(spec, q, k, W1, W2, ctl, phi_k, phi_q, y0):
    B, H, T, d = k.shape
    a = _lib.FeatureArgs()
    a.batch, a.heads, a.tokens, a.head_dim = B, H, T, d
    a.projections = W1.shape[1]
    a.kind = KINDS[spec.kind]
    a.basis = spec.basis
    a.bound = spec.bound
    a.eps = spec.eps
    a.k, a.q = k.data_ptr(), _ptr(q)
    a.k_strides = _lib.c_int64_3(*k.stride()[:3])
    if q is not None:
        a.q_strides = _lib.c_int64_3(*q.stride()[:3])
    a.w1, a.w2 = W1.data_ptr(), _ptr(W2)
    a.score_bias, a.threshold = _ptr(ctl["bias"]), _ptr(ctl["thr"])
    a.gain = _ptr(ctl["gain"])
    a.gain_per_feature = 1 if (ctl["gain"] is not None and ctl["gain"].ndim == 2) else 0
    a.gain_scalar = spec.gain
    a.spline_scale = _ptr(ctl["scale"])
    a.spline_scale_scalar = spec.spline_scale
    a.phi_k, a.phi_q, a.y0 = phi_k.data_ptr(), _ptr(phi_q), _ptr(y0)
    a.sparsity, a.threshold_temperature = SPARSITY[spec.sparsity], spec.temperature
    a.relative_threshold, a.sparse_blend = _ptr(ctl.get("rho")), _ptr(ctl.get("alpha"))
    return a


def _kread_args(spec, slots, eta, y0, y):
    B, H, T, d = y0.shape
    a = _lib.KReadArgs()
    a.batch, a.heads, a.tokens, a.head_dim = B, H, T, d
    a.mode = MODES[spec.mode]
    a.branches = len(slots) - 1
    a.eps = spec.eps
    for i, s in enumerate(slots):
        a.slots[i] = s.data_ptr()
    a.eta, a.y0, a.y = _ptr(eta), y0.data_ptr(), _ptr(y)
    a.mass_columns = MASS_COLS
    a.unnormalized = 0 if spec.read == "key_mass" else 1
    return a


def _slot_width(spec, d):
    """Columns of a scan read: [N | D | D] for the key-mass read, N otherwise."""
    return d + MASS_COLS if spec.read == "key_mass" else d


@dataclass(frozen=True)
class Prologue:
    """Row transform fused into the feature kernels: RoPE tables and L2 norm."""

    rot: int
    cos: torch.Tensor | None   # f32 [pos0 + T, rot/2]
    sin: torch.Tensor | None
    l2norm_eps: float | None   # None: no normalization
    pos0: int = 0              # sequence position of token 0 (sequence shards)


def _set_prologue(fa, prologue):
    if prologue is None:
        return
    fa.rope_rot = prologue.rot
    fa.rope_pos0 = prologue.pos0
    if prologue.rot:
        fa.rope_cos, fa.rope_sin = prologue.cos.data_ptr(), prologue.sin.data_ptr()
    if prologue.l2norm_eps is not None:
        fa.l2norm, fa.l2norm_eps = 1, prologue.l2norm_eps


def _controls(thr, bias, gain, scale, rho=None, alpha=None):
    return {"thr": _f32(thr), "bias": _f32(bias), "gain": _f32(gain), "scale": _f32(scale), "rho": _f32(rho),
            "alpha": _f32(alpha)}


def _stale_flags(spec, n_slots):
    """Slots 1..J of a stale bank are stale scans (the view S_sum - S_fast_j)."""
    return [False] + [True] * (n_slots - 1) if spec.mode == "stale" else None


def _core_forward(spec, q, k, v, W1, W2, ctl, log_alphas, etas, prologue):
    """Feature, scan and read kernels; returns y and what the backward needs."""
    lib = _lib.load()
    B, H, T, d = q.shape
    W1b = W1.detach().to(torch.bfloat16).contiguous()
    W2b = W2.detach().to(torch.bfloat16).contiguous()
    m = W1.shape[1] * (spec.basis if spec.kind == "projected_bspline" else 1)
    dev = q.device
    phi_k = torch.empty(B, H, T, m, dtype=torch.bfloat16, device=dev)
    phi_q = torch.empty_like(phi_k)
    y0 = torch.empty(B, H, T, d, dtype=torch.float32, device=dev)
    fa = _feature_args(spec, q, k, W1b, W2b, ctl, phi_k, phi_q, y0)
    _set_prologue(fa, prologue)
    _lib.check(lib.ts_b200_feature_fwd(ctypes.byref(fa), _stream()))

    las = [None] + ([] if log_alphas is None else
                    [log_alphas[j].detach().to(torch.float32).contiguous() for j in range(log_alphas.shape[0])])
    slots_all = torch.empty(len(las), B, H, T, d + MASS_COLS, dtype=torch.float32, device=dev)
    slots = list(slots_all.unbind(0))
    sa = _build_args(phi_q, phi_k, v, las, slots, MASS_COLS, stale=_stale_flags(spec, len(las)))
    ws = _workspace(lib, lib.ts_b200_scan_workspace_bytes, sa, dev)
    sa.workspace, sa.workspace_bytes = ws.data_ptr(), ws.numel()
    _lib.check(lib.ts_b200_scan_fwd(ctypes.byref(sa), _stream()))

    eta = None if etas is None else etas.detach().to(torch.float32).contiguous()
    y = torch.empty(B, T, H, d, dtype=torch.bfloat16, device=dev)
    ra = _kread_args(spec, slots, eta, y0, y)
    _lib.check(lib.ts_b200_kread_fwd(ctypes.byref(ra), _stream()))
    state = dict(W1b=W1b, W2b=W2b, phi_q=phi_q, phi_k=phi_k, ws=ws, slots=slots, slots_all=slots_all, las=las,
                 eta=eta, y0=y0)
    return y, state


def _saved_state(W1, W2, log_alphas, etas, phi_q, phi_k, y0, slots_all, ws):
    """The forward state of :func:`_core_forward` rebuilt from the tensors a
    forward op returned (the bf16 weight copies are made again)."""
    las = [None] + ([] if log_alphas is None else
                    [log_alphas[j].detach().to(torch.float32).contiguous() for j in range(log_alphas.shape[0])])
    eta = None if etas is None else etas.detach().to(torch.float32).contiguous()
    return dict(W1b=W1.detach().to(torch.bfloat16).contiguous(), W2b=W2.detach().to(torch.bfloat16).contiguous(),
                phi_q=phi_q, phi_k=phi_k, ws=ws, slots=list(slots_all.unbind(0)), las=las, eta=eta, y0=y0)


def _core_backward(spec, q, k, v, st, ctl, dy, prologue, dq_out, dk_out, dv_out):
    """Backward of the three stages.  ``dq_out``/``dk_out``/``dv_out`` are either
    ``None`` (fresh f32 dq, dk and a bf16 [.., d+1] dv are returned) or bf16
    strided views that receive the gradients in place."""
    lib = _lib.load()
    slots, las, eta, y0 = st["slots"], st["las"], st["eta"], st["y0"]
    W1b, W2b, phi_q, phi_k = st["W1b"], st["W2b"], st["phi_q"], st["phi_k"]
    n = len(slots)
    B, H, T, d = q.shape
    dev = q.device
    dy = dy.contiguous()
    if dy.dtype not in (torch.bfloat16, torch.float32):
        dy = dy.float()

    # 1. read epilogue
    ra = _kread_args(spec, slots, eta, y0, None)
    ga = _lib.KReadGradArgs()
    ga.dy = dy.data_ptr()
    ga.dy_dtype = _lib.TS_DTYPE_BF16 if dy.dtype == torch.bfloat16 else _lib.TS_DTYPE_F32
    dslots = [torch.empty(B, H, T, d + MASS_COLS, dtype=torch.bfloat16, device=dev) for _ in slots]
    for i, s in enumerate(dslots):
        ga.dslots[i] = s.data_ptr()
    # y0 enters y with coefficient 1, so its gradient is dy itself: a bf16 dy
    # is handed to the feature backward as a head-major view, an f32 one as the
    # head-major copy the read backward writes.
    dy0 = None
    if dy.dtype != torch.bfloat16:
        dy0 = torch.empty(B, H, T, d, dtype=torch.float32, device=dev)
        ga.dy0 = dy0.data_ptr()
    deta = torch.zeros(n - 1, H, dtype=torch.float32, device=dev) if n > 1 else None
    ga.deta = _ptr(deta)
    _lib.check(lib.ts_b200_kread_bwd(ctypes.byref(ra), ctypes.byref(ga), _stream()))

    # 2. scan
    sa = _build_args(phi_q, phi_k, v, las, slots, MASS_COLS, st["ws"], stale=_stale_flags(spec, n))
    sg = _lib.ScanGradArgs()
    m = phi_q.shape[-1]
    # bf16 hand-over: the feature backward stages dphi as a bf16 tile.
    dphi_q = torch.empty(B, H, T, m, dtype=torch.bfloat16, device=dev)
    dphi_k = torch.empty_like(dphi_q)
    if dv_out is None:
        dvaug = torch.empty(B, H, T, d + MASS_COLS, dtype=torch.bfloat16, device=dev)
        sg.dv = dvaug.data_ptr()
    else:
        dvaug = None
        sg.dv = dv_out.data_ptr()
        sg.dv_strides = _lib.c_int64_3(*dv_out.stride()[:3])
    dlas = [None] + [torch.zeros(H, dtype=torch.float32, device=dev) for _ in las[1:]]
    for i in range(n):
        sg.dout[i] = dslots[i].data_ptr()
        sg.dlog_alpha[i] = _ptr(dlas[i])
    sg.dq, sg.dk = dphi_q.data_ptr(), dphi_k.data_ptr()
    sg.grad_dtype = _lib.TS_DTYPE_BF16
    gws = _workspace(lib, lib.ts_b200_scan_bwd_workspace_bytes, sa, dev)
    sg.workspace, sg.workspace_bytes = gws.data_ptr(), gws.numel()
    _lib.check(lib.ts_b200_scan_bwd(ctypes.byref(sa), ctypes.byref(sg), _stream()))
    del gws

    # 3. features
    fa = _feature_args(spec, q, k, W1b, W2b, ctl, phi_k, phi_q, None)
    _set_prologue(fa, prologue)
    fg = _lib.FeatureGradArgs()
    fg.dphi_k, fg.dphi_q, fg.dphi_dtype = dphi_k.data_ptr(), dphi_q.data_ptr(), _lib.TS_DTYPE_BF16
    if dy0 is None:
        dyv = dy.permute(0, 2, 1, 3)
        fg.dy0_bf16 = dyv.data_ptr()
        fg.dy0_strides = _lib.c_int64_3(*dyv.stride()[:3])
    else:
        fg.dy0 = dy0.data_ptr()
    dq = dk = None
    if dq_out is None:
        dk = torch.empty(B, H, T, d, dtype=torch.float32, device=dev)
        dq = torch.empty_like(dk)
        fg.dk, fg.dq = dk.data_ptr(), dq.data_ptr()
    else:
        fg.dk_bf16, fg.dq_bf16 = dk_out.data_ptr(), dq_out.data_ptr()
        fg.dk_strides = _lib.c_int64_3(*dk_out.stride()[:3])
        fg.dq_strides = _lib.c_int64_3(*dq_out.stride()[:3])
    dW1 = torch.zeros(W1b.shape, dtype=torch.float32, device=dev)
    dW2t = torch.zeros(W2b.shape[0], W2b.shape[2], W2b.shape[1], dtype=torch.float32, device=dev)
    grads = {key: (torch.zeros_like(ctl[key]) if ctl[key] is not None else None)
             for key in ("thr", "bias", "gain", "scale", "rho", "alpha")}
    fg.dw1, fg.dw2, fg.dw2_transposed = dW1.data_ptr(), dW2t.data_ptr(), 1
    fg.dscore_bias, fg.dthreshold = _ptr(grads["bias"]), _ptr(grads["thr"])
    fg.dgain, fg.dspline_scale = _ptr(grads["gain"]), _ptr(grads["scale"])
    fg.drelative_threshold, fg.dsparse_blend = _ptr(grads["rho"]), _ptr(grads["alpha"])
    _lib.check(lib.ts_b200_feature_bwd(ctypes.byref(fa), ctypes.byref(fg), _stream()))
    dW2 = dW2t.transpose(1, 2)
    dla = None if n == 1 else torch.stack(dlas[1:])
    return dict(dq=dq, dk=dk, dvaug=dvaug, dW1=dW1, dW2=dW2, dla=dla, deta=deta, **grads)


def _qkv_views(qkv, H, d):
    B, T = qkv.shape[:2]
    q, k, v = qkv.view(B, T, 3, H, d).permute(2, 0, 3, 1, 4)
    return q, k, v


class _ShardScan:
    """What the two autograd stages of a sequence shard share: the scan
    workspaces (forward and backward), the slots and the entering state."""


def _features_fwd(spec, prologue, H, qkv, W1, W2, ctl):
    lib = _lib.load()
    d = qkv.shape[-1] // (3 * H)
    q, k, v = _qkv_views(qkv, H, d)
    B, _, T, _ = q.shape
    W1b = W1.detach().to(torch.bfloat16).contiguous()
    W2b = W2.detach().to(torch.bfloat16).contiguous()
    m = W1.shape[1] * (spec.basis if spec.kind == "projected_bspline" else 1)
    phi_k = torch.empty(B, H, T, m, dtype=torch.bfloat16, device=q.device)
    phi_q = torch.empty_like(phi_k)
    y0 = torch.empty(B, H, T, d, dtype=torch.float32, device=q.device)
    fa = _feature_args(spec, q, k, W1b, W2b, ctl, phi_k, phi_q, y0)
    _set_prologue(fa, prologue)
    _lib.check(lib.ts_b200_feature_fwd(ctypes.byref(fa), _stream()))
    return (q, k, v), W1b, W2b, phi_q, phi_k, y0


class _ShardStageA(torch.autograd.Function):
    """Features and the first half of the scan of one sequence shard: every
    tile's state and the shard total U (the state its tokens leave behind from
    a zero start).  Its backward finishes the scan backward from dU, the
    gradient the exchange hands back, then runs the feature backward."""

    @staticmethod
    def forward(ctx, hold, spec, prologue, H, qkv, W1, W2, thr, bias, gain, scale, log_alphas):
        lib = _lib.load()
        ctl = _controls(thr, bias, gain, scale)
        (q, k, v), W1b, W2b, phi_q, phi_k, y0 = _features_fwd(spec, prologue, H, qkv, W1, W2, ctl)
        B, _, T, d = q.shape
        m = phi_q.shape[-1]
        dev = q.device
        las = [None] + ([] if log_alphas is None else
                        [log_alphas[j].detach().to(torch.float32).contiguous() for j in range(log_alphas.shape[0])])
        R = len(las)
        slots = [torch.empty(B, H, T, d + MASS_COLS, dtype=torch.float32, device=dev) for _ in las]
        U = torch.empty(B, H, R, m, d + MASS_COLS, dtype=torch.float32, device=dev)
        sa = _build_args(phi_q, phi_k, v, las, slots, MASS_COLS)
        ws = _workspace(lib, lib.ts_b200_scan_workspace_bytes, sa, dev)
        sa.workspace, sa.workspace_bytes = ws.data_ptr(), ws.numel()
        sa.final_state, sa.stage = U.data_ptr(), 1
        _lib.check(lib.ts_b200_scan_fwd(ctypes.byref(sa), _stream()))
        hold.ws, hold.slots, hold.las, hold.phi_q, hold.phi_k = ws, slots, las, phi_q, phi_k
        hold.dlas = [None] + [torch.zeros(H, dtype=torch.float32, device=dev) for _ in las[1:]]
        ctx.hold, ctx.spec, ctx.prologue, ctx.H, ctx.ctl = hold, spec, prologue, H, ctl
        ctx.W = (W1b, W2b)
        ctx.dtypes = (W1.dtype, W2.dtype)
        ctx.save_for_backward(qkv)
        # phi_q / phi_k reach the second half only as its scan operands (no
        # gradient returns through them): no zero gradients are materialised
        ctx.mark_non_differentiable(phi_q, phi_k)
        ctx.set_materialize_grads(False)
        return phi_q, phi_k, y0, U

    @staticmethod
    def backward(ctx, dphi_q_out, dphi_k_out, dy0, dU):
        lib = _lib.load()
        (qkv,) = ctx.saved_tensors
        hold, H, spec = ctx.hold, ctx.H, ctx.spec
        d = qkv.shape[-1] // (3 * H)
        q, k, v = _qkv_views(qkv, H, d)
        B, _, T, _ = q.shape
        dev = q.device
        dqkv = torch.empty_like(qkv)
        dq, dk, dv = _qkv_views(dqkv, H, d)
        # scan, second half: reverse prefix from dU, then dq / dk / dv
        sa = _build_args(hold.phi_q, hold.phi_k, v, hold.las, hold.slots, MASS_COLS, hold.ws)
        sa.init_state, sa.stage = hold.S.data_ptr(), 2
        sg = _lib.ScanGradArgs()
        m = hold.phi_q.shape[-1]
        dphi_q = torch.empty(B, H, T, m, dtype=torch.bfloat16, device=dev)
        dphi_k = torch.empty_like(dphi_q)
        sg.dv = dv.data_ptr()
        sg.dv_strides = _lib.c_int64_3(*dv.stride()[:3])
        for i in range(len(hold.las)):
            sg.dout[i] = hold.douts[i].data_ptr()
            sg.dlog_alpha[i] = _ptr(hold.dlas[i])
        sg.dq, sg.dk = dphi_q.data_ptr(), dphi_k.data_ptr()
        sg.grad_dtype = _lib.TS_DTYPE_BF16
        sg.workspace, sg.workspace_bytes = hold.gws.data_ptr(), hold.gws.numel()
        if dU is None:
            dU = torch.zeros(B, H, len(hold.las), m, d + MASS_COLS, dtype=torch.float32, device=dev)
        dU = dU.float().contiguous()
        sg.dfinal_state = _ptr(dU)
        sg.stage = 2
        _lib.check(lib.ts_b200_scan_bwd(ctypes.byref(sa), ctypes.byref(sg), _stream()))
        del hold.gws
        if dphi_q_out is not None:
            dphi_q = (dphi_q.float() + dphi_q_out.float()).to(torch.bfloat16)
        if dphi_k_out is not None:
            dphi_k = (dphi_k.float() + dphi_k_out.float()).to(torch.bfloat16)
        # features
        W1b, W2b = ctx.W
        ctl = ctx.ctl
        fa = _feature_args(spec, q, k, W1b, W2b, ctl, hold.phi_k, hold.phi_q, None)
        _set_prologue(fa, ctx.prologue)
        fg = _lib.FeatureGradArgs()
        fg.dphi_k, fg.dphi_q, fg.dphi_dtype = dphi_k.data_ptr(), dphi_q.data_ptr(), _lib.TS_DTYPE_BF16
        if dy0 is None:
            dy0 = torch.zeros(B, H, T, d, dtype=torch.float32, device=dev)
        dy0 = dy0.float().contiguous()
        fg.dy0 = dy0.data_ptr()
        fg.dk_bf16, fg.dq_bf16 = dk.data_ptr(), dq.data_ptr()
        fg.dk_strides = _lib.c_int64_3(*dk.stride()[:3])
        fg.dq_strides = _lib.c_int64_3(*dq.stride()[:3])
        dW1 = torch.zeros(W1b.shape, dtype=torch.float32, device=dev)
        dW2t = torch.zeros(W2b.shape[0], W2b.shape[2], W2b.shape[1], dtype=torch.float32, device=dev)
        grads = {key: (torch.zeros_like(ctl[key]) if ctl[key] is not None else None)
                 for key in ("thr", "bias", "gain", "scale")}
        fg.dw1, fg.dw2, fg.dw2_transposed = dW1.data_ptr(), dW2t.data_ptr(), 1
        fg.dscore_bias, fg.dthreshold = _ptr(grads["bias"]), _ptr(grads["thr"])
        fg.dgain, fg.dspline_scale = _ptr(grads["gain"]), _ptr(grads["scale"])
        _lib.check(lib.ts_b200_feature_bwd(ctypes.byref(fa), ctypes.byref(fg), _stream()))
        dW2 = dW2t.transpose(1, 2)
        w1d, w2d = ctx.dtypes
        dla = None if len(hold.las) == 1 else torch.stack(hold.dlas[1:])
        return (None, None, None, None, dqkv, dW1.to(w1d), dW2.to(w2d), grads["thr"], grads["bias"],
                grads["gain"], grads["scale"], dla)


class _ShardStageB(torch.autograd.Function):
    """Second half of the scan forward of a shard and its key-mass read:
    carried states from the entering state S, the retention slots, then the
    read and bank blend into token-major ``y``.  Its backward runs the read
    backward and the first half of the scan backward (the slot gradients stay
    bf16 inside) and returns dS, the gradient of the entering state from this
    shard's own outputs, with d y0 and d eta."""

    @staticmethod
    def forward(ctx, hold, S, v, spec, y0, etas):
        lib = _lib.load()
        hold.S = S.detach().float().contiguous()
        sa = _build_args(hold.phi_q, hold.phi_k, v, hold.las, hold.slots, MASS_COLS, hold.ws)
        sa.init_state, sa.stage = hold.S.data_ptr(), 2
        _lib.check(lib.ts_b200_scan_fwd(ctypes.byref(sa), _stream()))
        B, H, T, d = y0.shape
        eta = None if etas is None else etas.detach().to(torch.float32).contiguous()
        y = torch.empty(B, T, H, d, dtype=torch.bfloat16, device=y0.device)
        ra = _kread_args(spec, hold.slots, eta, y0.contiguous(), y)
        _lib.check(lib.ts_b200_kread_fwd(ctypes.byref(ra), _stream()))
        ctx.hold, ctx.spec, ctx.eta, ctx.has_eta = hold, spec, eta, etas is not None
        ctx.save_for_backward(v, y0)
        return y

    @staticmethod
    def backward(ctx, dy):
        lib = _lib.load()
        hold = ctx.hold
        v, y0 = ctx.saved_tensors
        B, H, T, d = y0.shape
        dev = v.device
        dy = dy.contiguous()
        if dy.dtype not in (torch.bfloat16, torch.float32):
            dy = dy.float()
        ra = _kread_args(ctx.spec, hold.slots, ctx.eta, y0.contiguous(), None)
        ga = _lib.KReadGradArgs()
        ga.dy = dy.data_ptr()
        ga.dy_dtype = _lib.TS_DTYPE_BF16 if dy.dtype == torch.bfloat16 else _lib.TS_DTYPE_F32
        hold.douts = [torch.empty(B, H, T, _slot_width(ctx.spec, d), dtype=torch.bfloat16, device=dev)
                      for _ in hold.slots]
        for i, s_ in enumerate(hold.douts):
            ga.dslots[i] = s_.data_ptr()
        dy0 = torch.empty(B, H, T, d, dtype=torch.float32, device=dev)
        ga.dy0 = dy0.data_ptr()
        n = len(hold.slots)
        deta = torch.zeros(n - 1, H, dtype=torch.float32, device=dev) if n > 1 else None
        ga.deta = _ptr(deta)
        _lib.check(lib.ts_b200_kread_bwd(ctypes.byref(ra), ctypes.byref(ga), _stream()))
        sa = _build_args(hold.phi_q, hold.phi_k, v, hold.las, hold.slots, MASS_COLS, hold.ws)
        sa.init_state, sa.stage = hold.S.data_ptr(), 2
        hold.gws = _workspace(lib, lib.ts_b200_scan_bwd_workspace_bytes, sa, dev)
        sg = _lib.ScanGradArgs()
        for i in range(len(hold.las)):
            sg.dout[i] = hold.douts[i].data_ptr()
            sg.dlog_alpha[i] = _ptr(hold.dlas[i])
        # dq / dk / dv are written by the second half (stage A's backward)
        sg.grad_dtype = _lib.TS_DTYPE_BF16
        sg.workspace, sg.workspace_bytes = hold.gws.data_ptr(), hold.gws.numel()
        dS = torch.empty_like(hold.S)
        sg.dinit_state, sg.stage = dS.data_ptr(), 1
        _lib.check(lib.ts_b200_scan_bwd(ctypes.byref(sa), ctypes.byref(sg), _stream()))
        return None, dS, None, None, dy0, deta if ctx.has_eta else None


class _MassQuery(torch.autograd.Function):
    """``phi_q / (mass + eps)`` of one view (``ts_b200_mass_query_fwd``), the
    query of that view's unnormalized scan in the feature-mass read."""

    @staticmethod
    def _args(phi_k, phi_q, la, stale, eps, out, f32_quotient=False):
        """``phi_q`` bf16, or f32 (read instead, one rounding less); the
        quotient bf16, or unrounded f32 for a float32 scan."""
        B, H, T, m = phi_k.shape
        a = _lib.MassArgs()
        a.batch, a.heads, a.tokens, a.width = B, H, T, m
        a.phi_k = phi_k.data_ptr()
        if phi_q.dtype == torch.float32:
            a.phi_q_f32 = phi_q.data_ptr()
        else:
            a.phi_q = phi_q.data_ptr()
        a.log_alpha = _ptr(la)
        a.stale, a.eps = 1 if stale else 0, eps
        a.q_scaled = _ptr(out)
        a.q_scaled_f32 = 1 if f32_quotient else 0
        return a

    @staticmethod
    def forward(ctx, phi_k, phi_q, la, stale, eps):
        lib = _lib.load()
        la32 = None if la is None else la.detach().reshape(-1).to(torch.float32).contiguous()
        qn = torch.empty(phi_q.shape, dtype=torch.bfloat16, device=phi_q.device)
        a = _MassQuery._args(phi_k, phi_q, la32, stale, eps, qn)
        _lib.check(lib.ts_b200_mass_query_fwd(ctypes.byref(a), _stream()))
        ctx.stale, ctx.eps, ctx.la32 = stale, eps, la32
        ctx.la_meta = None if la is None else (la.dtype, la.shape)
        ctx.save_for_backward(phi_k, phi_q)
        return qn

    @staticmethod
    def backward(ctx, dqn):
        lib = _lib.load()
        phi_k, phi_q = ctx.saved_tensors
        a = _MassQuery._args(phi_k, phi_q, ctx.la32, ctx.stale, ctx.eps, None)
        dqn = dqn.contiguous()
        if dqn.dtype not in (torch.bfloat16, torch.float32):
            dqn = dqn.float()
        dphi_q = torch.zeros(phi_q.shape, dtype=torch.float32, device=phi_q.device)
        dphi_k = torch.zeros_like(dphi_q)
        dla = None if ctx.la32 is None else torch.zeros_like(ctx.la32)
        ws = _workspace(lib, lib.ts_b200_mass_query_bwd_workspace_bytes, a, phi_q.device)
        g = _lib.MassGradArgs()
        g.dq_scaled = dqn.data_ptr()
        g.dq_dtype = _lib.TS_DTYPE_BF16 if dqn.dtype == torch.bfloat16 else _lib.TS_DTYPE_F32
        g.dphi_q, g.dphi_k, g.dlog_alpha = dphi_q.data_ptr(), dphi_k.data_ptr(), _ptr(dla)
        g.workspace, g.workspace_bytes = ws.data_ptr(), ws.numel()
        _lib.check(lib.ts_b200_mass_query_bwd(ctypes.byref(a), ctypes.byref(g), _stream()))
        if dla is not None:
            dla = dla.to(ctx.la_meta[0]).reshape(ctx.la_meta[1])
        return dphi_k, dphi_q, dla, None, None


def _stale_f32_args(query, f32_kv, la, out, workspace=None):
    """Scan arguments of a stale feature-mass view on float32 streams: the
    f32 quotient against f32 copies of the bf16 keys and values, read as the
    plain sum and the decayed view (the stale read is their difference, as
    the reference forms it).  Returns the arguments and the decayed read to
    subtract from ``out``; in the backward (``workspace`` given) nothing is
    written and ``out`` only fills both output slots."""
    k32, v32 = f32_kv
    fast = out if workspace is not None else torch.empty_like(out)
    return _build_args(query, k32, v32, [None, la], [out, fast], 0, workspace), fast


class _KernelCoreViews(torch.autograd.Function):
    """Unnormalized and feature-mass reads (engine.py:402-416, 443-456) in one
    autograd stage, so that the gradients of phi_q and phi_k -- whose scan and
    mass parts nearly cancel under the feature-mass quotient -- are summed in
    f32 before the feature backward:

    forward   features -> [per view: phi_q / (mass_v + eps)] -> unnormalized
              scans (f32 reads) -> unnormalized blend
    backward  blend -> scans (f32 dq, dk, dv) -> mass backward -> features
    """

    @staticmethod
    def forward(ctx, spec, q, k, v, W1, W2, thr, bias, gain, scale, log_alphas, etas):
        lib = _lib.load()
        B, H, T, d = q.shape
        dev = q.device
        ctl = _controls(thr, bias, gain, scale)
        W1b = W1.detach().to(torch.bfloat16).contiguous()
        W2b = W2.detach().to(torch.bfloat16).contiguous()
        m = W1.shape[1] * (spec.basis if spec.kind == "projected_bspline" else 1)
        phi_k = torch.empty(B, H, T, m, dtype=torch.bfloat16, device=dev)
        phi_q = torch.empty_like(phi_k)
        y0 = torch.empty(B, H, T, d, dtype=torch.float32, device=dev)
        fa = _feature_args(spec, q, k, W1b, W2b, ctl, phi_k, phi_q, y0)
        # the feature-mass quotient reads phi(q) before its bf16 rounding
        phi_q32 = torch.empty(B, H, T, m, dtype=torch.float32, device=dev) if spec.read == "feature_mass" else None
        fa.phi_q_f32 = _ptr(phi_q32)
        _lib.check(lib.ts_b200_feature_fwd(ctypes.byref(fa), _stream()))
        J = 0 if log_alphas is None else log_alphas.shape[0]
        las = [None] + [log_alphas[j].detach().to(torch.float32).contiguous() for j in range(J)]
        flags = [False] + [spec.mode == "stale"] * J
        slots = [torch.empty(B, H, T, d, dtype=torch.float32, device=dev) for _ in las]
        if spec.read == "none":
            groups = [(phi_q, list(range(len(las))))]
        else:
            groups = []
            for i, la in enumerate(las):
                # a stale view's quotient stays f32 and its scan runs on f32 streams
                qn = torch.empty(B, H, T, m, dtype=torch.float32 if flags[i] else torch.bfloat16, device=dev)
                ma = _MassQuery._args(phi_k, phi_q32, la, flags[i], spec.eps, qn, f32_quotient=flags[i])
                _lib.check(lib.ts_b200_mass_query_fwd(ctypes.byref(ma), _stream()))
                groups.append((qn, [i]))
        scans = []
        f32_kv = None
        for query, idx in groups:
            if query.dtype == torch.float32:
                if f32_kv is None:
                    f32_kv = (phi_k.float(), v.float().contiguous())
                sa, extra = _stale_f32_args(query, f32_kv, las[idx[0]], slots[idx[0]])
            else:
                sa = _build_args(query, phi_k, v, [las[i] for i in idx], [slots[i] for i in idx], 0,
                                 stale=[flags[i] for i in idx])
                extra = None
            ws = _workspace(lib, lib.ts_b200_scan_workspace_bytes, sa, dev)
            sa.workspace, sa.workspace_bytes = ws.data_ptr(), ws.numel()
            _lib.check(lib.ts_b200_scan_fwd(ctypes.byref(sa), _stream()))
            if extra is not None:
                slots[idx[0]].sub_(extra)
            scans.append((query, idx, ws))
        eta = None if etas is None else etas.detach().to(torch.float32).contiguous()
        y = torch.empty(B, T, H, d, dtype=torch.bfloat16, device=dev)
        ra = _kread_args(spec, slots, eta, y0, y)
        _lib.check(lib.ts_b200_kread_fwd(ctypes.byref(ra), _stream()))
        ctx.spec, ctx.ctl, ctx.W, ctx.las, ctx.flags = spec, ctl, (W1b, W2b), las, flags
        ctx.scans, ctx.slots, ctx.eta, ctx.y0 = scans, slots, eta, y0
        ctx.phi = (phi_q, phi_k, phi_q32)
        ctx.f32_kv = f32_kv
        ctx.dtypes = (q.dtype, k.dtype, v.dtype, W1.dtype, W2.dtype)
        ctx.has_eta = etas is not None
        ctx.save_for_backward(q, k, v)
        return y

    @staticmethod
    def backward(ctx, dy):
        lib = _lib.load()
        q, k, v = ctx.saved_tensors
        spec, las, flags, slots = ctx.spec, ctx.las, ctx.flags, ctx.slots
        phi_q, phi_k, phi_q32 = ctx.phi
        W1b, W2b = ctx.W
        B, H, T, d = q.shape
        m = phi_q.shape[-1]
        dev = q.device
        dy = dy.contiguous()
        if dy.dtype not in (torch.bfloat16, torch.float32):
            dy = dy.float()
        # 1. blend
        ra = _kread_args(spec, slots, ctx.eta, ctx.y0, None)
        ga = _lib.KReadGradArgs()
        ga.dy = dy.data_ptr()
        ga.dy_dtype = _lib.TS_DTYPE_BF16 if dy.dtype == torch.bfloat16 else _lib.TS_DTYPE_F32
        dslots = [torch.empty(B, H, T, d, dtype=torch.bfloat16, device=dev) for _ in slots]
        for i, t in enumerate(dslots):
            ga.dslots[i] = t.data_ptr()
        dy0 = torch.empty(B, H, T, d, dtype=torch.float32, device=dev)
        ga.dy0 = dy0.data_ptr()
        n = len(slots)
        deta = torch.zeros(n - 1, H, dtype=torch.float32, device=dev) if n > 1 else None
        ga.deta = _ptr(deta)
        _lib.check(lib.ts_b200_kread_bwd(ctypes.byref(ra), ctypes.byref(ga), _stream()))
        # 2. scans (f32 gradients), then the mass of each view
        dphi_q = torch.zeros(B, H, T, m, dtype=torch.float32, device=dev)
        dphi_k = torch.zeros_like(dphi_q)
        dv = torch.zeros(B, H, T, d, dtype=torch.float32, device=dev)
        dlas = [None] + [torch.zeros(H, dtype=torch.float32, device=dev) for _ in las[1:]]
        for query, idx, ws in ctx.scans:
            sg = _lib.ScanGradArgs()
            if query.dtype == torch.float32:
                # sum - fast: the fast slot's read gradient is -dslot, which
                # also gives its log-retention gradient the stale view's sign
                i = idx[0]
                sa, _ = _stale_f32_args(query, ctx.f32_kv, las[i], slots[i], ws)
                dsum = dslots[i].float()
                dfast = -dsum
                sg.dout[0], sg.dout[1] = dsum.data_ptr(), dfast.data_ptr()
                sg.dlog_alpha[1] = _ptr(dlas[i])
            else:
                sa = _build_args(query, phi_k, v, [las[i] for i in idx], [slots[i] for i in idx], 0, ws,
                                 stale=[flags[i] for i in idx])
                for j, i in enumerate(idx):
                    sg.dout[j] = dslots[i].data_ptr()
                    sg.dlog_alpha[j] = _ptr(dlas[i])
            dq_s = torch.empty(B, H, T, m, dtype=torch.float32, device=dev)
            dk_s = torch.empty_like(dq_s)
            dv_s = torch.empty(B, H, T, d, dtype=torch.float32, device=dev)
            sg.dq, sg.dk, sg.dv = dq_s.data_ptr(), dk_s.data_ptr(), dv_s.data_ptr()
            sg.grad_dtype = _lib.TS_DTYPE_F32
            gws = _workspace(lib, lib.ts_b200_scan_bwd_workspace_bytes, sa, dev)
            sg.workspace, sg.workspace_bytes = gws.data_ptr(), gws.numel()
            _lib.check(lib.ts_b200_scan_bwd(ctypes.byref(sa), ctypes.byref(sg), _stream()))
            del gws
            dphi_k += dk_s
            dv += dv_s
            if spec.read == "none":
                dphi_q += dq_s
                continue
            i = idx[0]
            ma = _MassQuery._args(phi_k, phi_q32, las[i], flags[i], spec.eps, None, f32_quotient=flags[i])
            mg = _lib.MassGradArgs()
            mg.dq_scaled, mg.dq_dtype = dq_s.data_ptr(), _lib.TS_DTYPE_F32
            mg.dphi_q, mg.dphi_k, mg.dlog_alpha = dphi_q.data_ptr(), dphi_k.data_ptr(), _ptr(dlas[i])
            mws = _workspace(lib, lib.ts_b200_mass_query_bwd_workspace_bytes, ma, dev)
            mg.workspace, mg.workspace_bytes = mws.data_ptr(), mws.numel()
            _lib.check(lib.ts_b200_mass_query_bwd(ctypes.byref(ma), ctypes.byref(mg), _stream()))
        # 3. features
        ctl = ctx.ctl
        fa = _feature_args(spec, q, k, W1b, W2b, ctl, phi_k, phi_q, None)
        fg = _lib.FeatureGradArgs()
        fg.dphi_k, fg.dphi_q, fg.dphi_dtype = dphi_k.data_ptr(), dphi_q.data_ptr(), _lib.TS_DTYPE_F32
        fg.dy0 = dy0.data_ptr()
        dk = torch.empty(B, H, T, d, dtype=torch.float32, device=dev)
        dq = torch.empty_like(dk)
        fg.dk, fg.dq = dk.data_ptr(), dq.data_ptr()
        dW1 = torch.zeros(W1b.shape, dtype=torch.float32, device=dev)
        dW2t = torch.zeros(W2b.shape[0], W2b.shape[2], W2b.shape[1], dtype=torch.float32, device=dev)
        grads = {key: (torch.zeros_like(ctl[key]) if ctl[key] is not None else None)
                 for key in ("thr", "bias", "gain", "scale")}
        fg.dw1, fg.dw2, fg.dw2_transposed = dW1.data_ptr(), dW2t.data_ptr(), 1
        fg.dscore_bias, fg.dthreshold = _ptr(grads["bias"]), _ptr(grads["thr"])
        fg.dgain, fg.dspline_scale = _ptr(grads["gain"]), _ptr(grads["scale"])
        _lib.check(lib.ts_b200_feature_bwd(ctypes.byref(fa), ctypes.byref(fg), _stream()))
        dW2 = dW2t.transpose(1, 2)
        qd, kd, vd, w1d, w2d = ctx.dtypes
        dla = None if n == 1 else torch.stack(dlas[1:])
        return (None, dq.to(qd), dk.to(kd), dv.to(vd), dW1.to(w1d), dW2.to(w2d), grads["thr"], grads["bias"],
                grads["gain"], grads["scale"], dla, deta if ctx.has_eta else None)


def kernel_core_sharded(qkv, H, W1, W2, spec: KernelSpec, prologue: Prologue | None, shard, *, threshold=None,
                        score_bias=None, gain=None, spline_scale=None, log_alphas=None, etas=None,
                        relative_threshold=None, sparse_blend=None):
    """The hot path of :func:`kernel_core_qkv` on one contiguous shard of the
    sequence (``prologue.pos0`` = its first position).  The scan runs in two
    halves around one exchange of shard totals (``shard.gather``, an
    all-gather on a process group): the first half leaves every tile's state
    and the shard total U; the entering state S is the decayed exclusive
    prefix of the earlier shards' totals (:func:`thetascan_b200.seqpar.entering_state`);
    the second half carries the states from S and reads.  The backward mirrors
    it: dS of every shard, the reverse exchange (all_gather's backward), then
    dq / dk / dv from each shard's dU."""
    from .seqpar import entering_state
    if not qkv.is_cuda:
        raise RuntimeError("b200 backend requires CUDA tensors")
    if qkv.dtype != torch.bfloat16 or qkv.dim() != 3 or not qkv.is_contiguous():
        raise ValueError("kernel_core_sharded: qkv must be a contiguous bf16 [B,T,3*H*d] tensor")
    if (log_alphas is None) != (spec.mode == "sum"):
        raise ValueError("kernel_core_sharded: log_alphas are required exactly for a bank (mode fast/stale)")
    if spec.mode == "stale":
        raise NotImplementedError("b200 backend: sequence shards of a stale bank are not built (stale scans take "
                                  "no boundary states); fast banks and the plain sum shard")
    if spec.read != "key_mass" or spec.sparsity != "none":
        raise NotImplementedError("b200 backend: sequence shards read with key mass and no relative sparsity only")
    hold = _ShardScan()
    phi_q, phi_k, y0, U = _ShardStageA.apply(hold, spec, prologue, H, qkv, W1, W2, threshold, score_bias, gain,
                                             spline_scale, log_alphas)
    totals = shard.gather(U)
    las = [None] + ([] if log_alphas is None else [log_alphas[j] for j in range(log_alphas.shape[0])])
    S = entering_state(totals, las, qkv.shape[1], shard.rank)
    if shard.rank == 0:
        # a zero state, but the graph must reach the gather: its backward is a
        # collective every rank joins
        S = S + 0.0 * totals[0]
    d = qkv.shape[-1] // (3 * H)
    return _ShardStageB.apply(hold, S, _qkv_views(qkv, H, d)[2], spec, y0, etas)


def kernel_core_qkv(qkv, H, W1, W2, spec: KernelSpec, prologue: Prologue | None, *, threshold=None,
                    score_bias=None, gain=None, spline_scale=None, log_alphas=None, etas=None,
                    relative_threshold=None, sparse_blend=None):
    """Hot path from the raw fused projection; returns ``y`` token-major ``[B,T,H,d]``.

    ``qkv``: bf16 ``[B,T,3*H*d]`` output of the fused q/k/v projection
    (block.py:593-594 layout: q, k, v blocks of ``H*d``).  ``prologue``
    applies RoPE and the L2 norm to q and k inside the feature kernels, as
    block.py:595-599 does before the mixer core."""
    if not qkv.is_cuda:
        raise RuntimeError("b200 backend requires CUDA tensors")
    if qkv.dtype != torch.bfloat16 or qkv.dim() != 3 or not qkv.is_contiguous():
        raise ValueError("kernel_core_qkv: qkv must be a contiguous bf16 [B,T,3*H*d] tensor")
    if qkv.shape[-1] % (3 * H):
        raise ValueError("kernel_core_qkv: last dimension must be 3*H*d")
    if (log_alphas is None) != (spec.mode == "sum"):
        raise ValueError("kernel_core_qkv: log_alphas are required exactly for a bank (mode fast/stale)")
    if spec.read != "key_mass":
        raise NotImplementedError("kernel_core_qkv: the fused projection path reads with key mass; use kernel_core")
    from . import ops  # noqa: F401  (registers the operators)
    rot = prologue.rot if prologue is not None else 0
    outs = torch.ops.thetascan_b200.kernel_mixer_qkv_fwd(
        qkv, W1, W2, threshold, score_bias, gain, spline_scale, relative_threshold, sparse_blend, log_alphas, etas,
        prologue.cos if rot else None, prologue.sin if rot else None, H, rot,
        -1.0 if prologue is None or prologue.l2norm_eps is None else float(prologue.l2norm_eps),
        spec.kind, spec.mode, float(spec.eps), float(spec.gain), int(spec.basis), float(spec.bound),
        float(spec.spline_scale), spec.sparsity, float(spec.temperature))
    return outs[0]


def kernel_core(q, k, v, W1, W2, spec: KernelSpec, *, threshold=None, score_bias=None, gain=None,
                spline_scale=None, log_alphas=None, etas=None, relative_threshold=None, sparse_blend=None):
    """Kernel-family hot path on the GPU; returns ``y`` token-major ``[B,T,H,d]``.

    ``q, k, v``: bf16 ``[B,H,T,d]`` after RoPE / L2 norm.  ``W1 [H,P,d]`` and
    ``W2 [H,d,m]``: effective weights.  ``log_alphas``/``etas``: ``[J,H]`` for a
    bank (``spec.mode`` fast or stale), ``None`` for the plain sum.  The result
    equals ``q + W2 phi(q) + blended key-mass read`` of the reference (see
    the module docstring) up to bf16 rounding.
    """
    for x in (q, k, v):
        if not x.is_cuda:
            raise RuntimeError("b200 backend requires CUDA tensors")
        if x.dtype != torch.bfloat16:
            raise NotImplementedError("b200 backend: bf16 streams only")
        if x.stride(-1) != 1:
            raise ValueError("b200 backend: streams need a contiguous innermost dimension")
    if (log_alphas is None) != (spec.mode == "sum"):
        raise ValueError("kernel_core: log_alphas are required exactly for a bank (mode fast/stale)")
    if spec.read not in ("key_mass", "feature_mass", "none"):
        raise ValueError(f"kernel_core: unknown read normalization {spec.read!r}")
    if spec.read != "key_mass":
        if spec.sparsity != "none":
            raise NotImplementedError("b200 backend: relative sparsity reads with key mass only")
        return _KernelCoreViews.apply(spec, q, k, v, W1, W2, threshold, score_bias, gain, spline_scale,
                                      log_alphas, etas)
    from . import ops  # noqa: F401  (registers the operators)
    outs = torch.ops.thetascan_b200.kernel_mixer_fwd(
        q, k, v, W1, W2, threshold, score_bias, gain, spline_scale, relative_threshold, sparse_blend, log_alphas,
        etas, spec.kind, spec.mode, float(spec.eps), float(spec.gain), int(spec.basis), float(spec.bound),
        float(spec.spline_scale), spec.sparsity, float(spec.temperature))
    return outs[0]
