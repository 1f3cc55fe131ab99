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
    return a


class _KernelCore(torch.autograd.Function):
    @staticmethod
    def forward(ctx, spec, q, k, v, W1, W2, thr, bias, gain, scale, log_alphas, etas):
        lib = _lib.load()
        B, H, T, d = q.shape
        W1b = W1.detach().to(torch.bfloat16).contiguous()
        W2b = W2.detach().to(torch.bfloat16).contiguous()
        ctl = {"thr": _f32(thr), "bias": _f32(bias), "gain": _f32(gain), "scale": _f32(scale)}
        m = W1.shape[1] * (spec.basis if spec.kind == "projected_bspline" else 1)
        dev = q.device
        phi_k = torch.empty(B, H, T, m, dtype=torch.bfloat16, device=dev)
        phi_q = torch.empty_like(phi_k)
        y0 = torch.empty(B, H, T, d, dtype=torch.float32, device=dev)
        fa = _feature_args(spec, q, k, W1b, W2b, ctl, phi_k, phi_q, y0)
        _lib.check(lib.ts_b200_feature_fwd(ctypes.byref(fa), _stream()))

        las = [None] + ([] if log_alphas is None else
                        [log_alphas[j].detach().to(torch.float32).contiguous() for j in range(log_alphas.shape[0])])
        slots = [torch.empty(B, H, T, d + 1, dtype=torch.float32, device=dev) for _ in las]
        sa = _build_args(phi_q, phi_k, v, las, slots, True)
        ws = _workspace(lib, lib.ts_b200_scan_workspace_bytes, sa, dev)
        sa.workspace, sa.workspace_bytes = ws.data_ptr(), ws.numel()
        _lib.check(lib.ts_b200_scan_fwd(ctypes.byref(sa), _stream()))

        eta = None if etas is None else etas.detach().to(torch.float32).contiguous()
        y = torch.empty(B, T, H, d, dtype=torch.bfloat16, device=dev)
        ra = _kread_args(spec, slots, eta, y0, y)
        _lib.check(lib.ts_b200_kread_fwd(ctypes.byref(ra), _stream()))

        ctx.spec = spec
        ctx.has = (thr is not None, bias is not None, gain is not None, scale is not None,
                   log_alphas is not None)
        ctx.dtypes = (q.dtype, k.dtype, v.dtype, W1.dtype, W2.dtype)
        saved_las = [la for la in las[1:]]
        ctx.save_for_backward(q, k, v, W1b, W2b, phi_q, phi_k, ws, *slots, *saved_las,
                              *[t if t is not None else torch.empty(0, device=dev) for t in
                                (ctl["thr"], ctl["bias"], ctl["gain"], ctl["scale"], eta, y0)])
        ctx.n_slots = len(slots)
        return y

    @staticmethod
    def backward(ctx, dy):
        lib = _lib.load()
        spec = ctx.spec
        n = ctx.n_slots
        saved = ctx.saved_tensors
        q, k, v, W1b, W2b, phi_q, phi_k, ws = saved[:8]
        slots = list(saved[8:8 + n])
        las = [None] + list(saved[8 + n:8 + 2 * n - 1])
        thr, bias, gain, scale, eta, y0 = saved[8 + 2 * n - 1:]
        has_thr, has_bias, has_gain, has_scale, has_la = ctx.has
        thr = thr if has_thr else None
        bias = bias if has_bias else None
        gain = gain if has_gain else None
        scale = scale if has_scale else None
        eta = eta if has_la else None
        B, H, T, d = q.shape
        dev = q.device
        dy = dy.contiguous()

        # 1. read epilogue
        ra = _kread_args(spec, slots, eta, y0, None)
        ga = _lib.KReadGradArgs()
        ga.dy = dy.data_ptr()
        ga.dy_dtype = _lib.TS_DTYPE_BF16 if dy.dtype == torch.bfloat16 else _lib.TS_DTYPE_F32
        if dy.dtype not in (torch.bfloat16, torch.float32):
            dy = dy.float()
            ga.dy, ga.dy_dtype = dy.data_ptr(), _lib.TS_DTYPE_F32
        dslots = [torch.empty(B, H, T, d + 1, dtype=torch.bfloat16, device=dev) for _ in slots]
        for i, s in enumerate(dslots):
            ga.dslots[i] = s.data_ptr()
        dy0 = torch.empty(B, H, T, d, dtype=torch.float32, device=dev)
        ga.dy0 = dy0.data_ptr()
        deta = torch.zeros(n - 1, H, dtype=torch.float32, device=dev) if n > 1 else None
        ga.deta = _ptr(deta)
        _lib.check(lib.ts_b200_kread_bwd(ctypes.byref(ra), ctypes.byref(ga), _stream()))

        # 2. scan
        sa = _build_args(phi_q, phi_k, v, las, slots, True, ws)
        sg = _lib.ScanGradArgs()
        m = phi_q.shape[-1]
        # bf16 hand-over: the feature backward stages dphi as a bf16 tile.
        dphi_q = torch.empty(B, H, T, m, dtype=torch.bfloat16, device=dev)
        dphi_k = torch.empty_like(dphi_q)
        dvaug = torch.empty(B, H, T, d + 1, dtype=torch.bfloat16, device=dev)
        dlas = [None] + [torch.zeros(H, dtype=torch.float32, device=dev) for _ in las[1:]]
        for i in range(n):
            sg.dout[i] = dslots[i].data_ptr()
            sg.dlog_alpha[i] = _ptr(dlas[i])
        sg.dq, sg.dk, sg.dv = dphi_q.data_ptr(), dphi_k.data_ptr(), dvaug.data_ptr()
        sg.grad_dtype = _lib.TS_DTYPE_BF16
        gws = _workspace(lib, lib.ts_b200_scan_bwd_workspace_bytes, sa, dev)
        sg.workspace, sg.workspace_bytes = gws.data_ptr(), gws.numel()
        _lib.check(lib.ts_b200_scan_bwd(ctypes.byref(sa), ctypes.byref(sg), _stream()))
        del gws

        # 3. features
        ctl = {"thr": thr, "bias": bias, "gain": gain, "scale": scale}
        fa = _feature_args(spec, q, k, W1b, W2b, ctl, phi_k, phi_q, None)
        fg = _lib.FeatureGradArgs()
        fg.dphi_k, fg.dphi_q, fg.dphi_dtype = dphi_k.data_ptr(), dphi_q.data_ptr(), _lib.TS_DTYPE_BF16
        fg.dy0 = dy0.data_ptr()
        dk = torch.empty(B, H, T, d, dtype=torch.float32, device=dev)
        dq = torch.empty_like(dk)
        dW1 = torch.zeros(W1b.shape, dtype=torch.float32, device=dev)
        dW2 = torch.zeros(W2b.shape, dtype=torch.float32, device=dev)
        dthr = torch.zeros_like(thr) if thr is not None else None
        dbias = torch.zeros_like(bias) if bias is not None else None
        dgain = torch.zeros_like(gain) if gain is not None else None
        dscale = torch.zeros_like(scale) if scale is not None else None
        fg.dk, fg.dq, fg.dw1, fg.dw2 = dk.data_ptr(), dq.data_ptr(), dW1.data_ptr(), dW2.data_ptr()
        fg.dscore_bias, fg.dthreshold = _ptr(dbias), _ptr(dthr)
        fg.dgain, fg.dspline_scale = _ptr(dgain), _ptr(dscale)
        _lib.check(lib.ts_b200_feature_bwd(ctypes.byref(fa), ctypes.byref(fg), _stream()))

        qd, kd, vd, w1d, w2d = ctx.dtypes
        dla = None if n == 1 else torch.stack(dlas[1:])
        return (None, dq.to(qd), dk.to(kd), dvaug[..., :d].to(vd), dW1.to(w1d), dW2.to(w2d),
                dthr, dbias, dgain, dscale, dla, deta)


def kernel_core(q, k, v, W1, W2, spec: KernelSpec, *, threshold=None, score_bias=None, gain=None,
                spline_scale=None, log_alphas=None, etas=None):
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
    if spec.mode == "stale":
        raise NotImplementedError(
            "b200 backend: the stale bank reads a difference of two scans whose mass can vanish; "
            "its dedicated retention kind is not built yet (fast banks are supported)")
    return _KernelCore.apply(spec, q, k, v, W1, W2, threshold, score_bias, gain, spline_scale, log_alphas, etas)
