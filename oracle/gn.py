"""Gauss--Newton (GN) family of the mixer hot path: float64 CPU restatement.

Test infrastructure only (the checker of the GPU path, never shipped or
measured).  One memory block (depth 1) with one Jacobian step, as the
reference runs it for ``family="gn"`` (src/thetascan/config.py:745-756):

write (engine.write_streams, src/thetascan/_core/ops/engine.py:260-340):
  a = W1 k, pre = rmsnorm(a) [- tau], h = sigma(pre), o = k + W2 h,
  r = v - o,
  lambda = r / (||h||^2 + ||k||^2 (W2^2)(s^2) + eps),  s = sigma'(pre) / rms(a)
                                                  (_lambda_solve, engine.py:215-255)
  g = sigma'(pre) (W2^T lambda) / rms(a)          (_g_from_lambda, engine.py:180-195)
  streams LA1 = (k, g), LA2 = (h, lambda)

read (engine.dual_read_views.layer, engine.py:455-528), per temporal view:
  two-stage (read_norm_w1): h0 = relu2(rmsnorm(W1 q) [- tau]),
      c = scan(h0; h, [g | 1]), pre = W1 q + c[:m] / (c[m] + eps)
  otherwise: pre = W1 q + scan(q; k, g)
  h_q = sigma(rmsnorm(pre) [- tau]), base = W2 h_q,
  mem = scan(h_q; h, [lambda | 1]) normalized (read_norm) or scan(h_q; h, lambda),
  y_view = q + base + mem;
views blended like the kernel family (block.py:676-718); a stale bank
subtracts eta_j (y_stale_j - y_base), y_base the zero-memory read
q + W2 sigma(rmsnorm(W1 q) [- tau]) (block.py:697-718).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from . import features, scan


def activation(nonlin: str, pre: torch.Tensor) -> torch.Tensor:
    """sigma (reference nonlin.py:13-31)."""
    if nonlin == "relu2":
        r = F.relu(pre)
        return r * r
    if nonlin == "silu":
        return F.silu(pre)
    if nonlin == "tanh":
        # extension (config 3 as the baseline states it): an entry of the
        # reference's ELEMENTWISE table (nonlin.py:28-31), tanh / 1 - h^2
        return torch.tanh(pre)
    raise ValueError(f"unsupported GN nonlinearity: {nonlin!r}")


def activation_grad(nonlin: str, pre: torch.Tensor) -> torch.Tensor:
    """sigma' (reference nonlin.py:18-26)."""
    if nonlin == "relu2":
        return 2.0 * F.relu(pre)
    if nonlin == "silu":
        s = torch.sigmoid(pre)
        return s * (1 + pre * (1 - s))
    if nonlin == "tanh":
        h = torch.tanh(pre)
        return 1.0 - h * h
    raise ValueError(f"unsupported GN nonlinearity: {nonlin!r}")


def _thresholded(pre, tau):
    """Subtract the learned per-unit threshold (engine.py:127-134)."""
    return pre if tau is None else pre - tau[..., 0].unsqueeze(0).unsqueeze(2).to(pre.dtype)


def gn_write(k, v, W1, W2, tau, nonlin: str, eps: float):
    """(h, g, lambda) of every token; W1 ``[H,m,d]``, W2 ``[H,d,m]``, tau ``[H,m,1]``."""
    a = torch.einsum("hmd,bhtd->bhtm", W1, k)
    pre, inv = features.rmsnorm(a, eps)
    pre = _thresholded(pre, tau)
    h = activation(nonlin, pre)
    o = k + torch.einsum("hdm,bhtm->bhtd", W2, h)
    r = v - o
    dsig = activation_grad(nonlin, pre)
    s = dsig * inv
    rowsq = torch.einsum("hdm,bhtm->bhtd", W2 * W2, s * s)
    diag = (h * h).sum(-1, keepdim=True) + (k * k).sum(-1, keepdim=True) * rowsq
    lam = r / (diag + eps)
    g = dsig * torch.einsum("hdm,bhtd->bhtm", W2, lam) * inv
    return h, g, lam


def _combine(scanned, view):
    total = None
    for coef, slot in view:
        piece = scanned[slot] if coef == 1.0 else coef * scanned[slot]
        total = piece if total is None else total + piece
    return total


def gn_core(q, k, v, W1, W2, tau, *, nonlin: str, read_norm: bool, read_norm_w1: bool,
            log_alphas=None, etas=None, mode: str = "fast", eps: float = 1e-6, chunk: int = 512,
            scan_fn=None):
    """GN mixer core ``[B,H,T,d]`` (q, k after RoPE / L2 norm) with its temporal views."""
    from .mixer import blend_outputs, view_terms
    if scan_fn is None:
        scan_fn = lambda qq, kk, vv, rets: scan.linattn_chunk_views(qq, kk, vv, rets, chunk)
    m = W1.shape[1]
    h_k, g, lam = gn_write(k, v, W1, W2, tau, nonlin, eps)
    J = 0 if log_alphas is None else log_alphas.shape[0]
    retentions = tuple([None] + [log_alphas[j] for j in range(J)])
    terms = view_terms(mode, J)
    a = torch.einsum("hmd,bhtd->bhtm", W1, q)
    # stage 1: the hidden correction of every view
    if read_norm_w1:
        h0 = activation("relu2", _thresholded(features.rmsnorm(a, eps)[0], tau))
        unit = torch.cat([g, g.new_ones(*g.shape[:3], 1)], dim=-1)
        scanned = scan_fn(h0.to(h_k.dtype), h_k, unit, retentions)
        pres = []
        for view in terms:
            c = _combine(scanned, view)
            pres.append(a + c[..., :m] / (c[..., -1:] + eps))
    else:
        scanned = scan_fn(q, k, g, retentions)
        pres = [a + _combine(scanned, view) for view in terms]
    # stage 2: each view's own query
    outs, base_out = [], None
    for view, pre in zip(terms, pres):
        hq = activation(nonlin, _thresholded(features.rmsnorm(pre, eps)[0], tau))
        base = torch.einsum("hdm,bhtm->bhtd", W2, hq)
        if read_norm:
            unit = torch.cat([lam, lam.new_ones(*lam.shape[:3], 1)], dim=-1)
            c = _combine(scan_fn(hq.to(h_k.dtype), h_k, unit, retentions), view)
            mem = c[..., :-1] / (c[..., -1:] + eps)
        else:
            mem = _combine(scan_fn(hq.to(h_k.dtype), h_k, lam, retentions), view)
        outs.append(q + base + mem)
    if J and mode == "stale":
        # the zero-memory read of the stale blend (NullAccumulator, interface.py:
        # 310-327): every scan is zero, so pre = W1 q and mem = 0
        h_base = activation(nonlin, _thresholded(features.rmsnorm(a, eps)[0], tau))
        base_out = q + torch.einsum("hdm,bhtm->bhtd", W2, h_base)
    return blend_outputs(outs, base_out, mode, etas) if J else outs[0]
