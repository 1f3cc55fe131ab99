"""Gauss--Newton (GN) family of the mixer hot path: float64 CPU restatement.

Test infrastructure only (the checker of the GPU path, never shipped or
measured).  ``gn_core``: one memory block (depth 1) with one Jacobian step,
as the reference runs it for ``family="gn"`` (src/thetascan/config.py:745-756);
``gn_core_net`` (end of the file): nets of any depth, the swiglu activation
and two Jacobian steps.  The one-block form:

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


# --------------------------------------------------------------------------- nets of any depth, swiglu, two steps
#
# The general GN memory net of the reference engine (engine.py:117-340,
# 345-544): L blocks with the residual x_{l+1} = x_l + u_l / sqrt(L), the
# swiglu activation h = silu(rms(Wg x)) * rms(W1 x) (nonlin.py:34-37 for
# silu'), the Jacobi diagonal summed over the blocks, one or two Jacobian
# steps (write_iters), and the per-layer read of every view.  Each view is
# evaluated on its own here (the reference shares the first layer's scans
# between views, which changes nothing numerically).

def _net_features(a, b, Wg, nonlin, learn_thresh, eps):
    """(pre, h, inv_a, preb, inv_b) of one block (engine.py:117-158)."""
    pre, inv_a = features.rmsnorm(a, eps)
    if nonlin == "swiglu":
        preb, inv_b = features.rmsnorm(b, eps)
        return pre, F.silu(preb) * pre, inv_a, preb, inv_b
    if learn_thresh:
        pre = _thresholded(pre, Wg)
    return pre, activation(nonlin, pre), inv_a, None, None


def _net_block(layer, x, nonlin, learn_thresh, eps, delta=None):
    """u = W2 h and the block's activations; ``delta`` = (x0, h0, lam_hat, g)
    is the token's own first-step write (engine.py:117-158)."""
    W1, W2, Wg = layer
    a = torch.einsum("hmd,bhtd->bhtm", W1, x)
    b = torch.einsum("hmd,bhtd->bhtm", Wg, x) if nonlin == "swiglu" else None
    if delta is not None:
        x0, h0, lam_hat, g = delta
        xx = (x0 * x).sum(-1, keepdim=True)
        m = a.shape[-1]
        a = a + g[..., :m] * xx
        if b is not None:
            b = b + g[..., m:] * xx
    pre, h, inv_a, preb, inv_b = _net_features(a, b, Wg, nonlin, learn_thresh, eps)
    u = torch.einsum("hdm,bhtm->bhtd", W2, h)
    if delta is not None:
        u = u + delta[2] * (delta[1] * h).sum(-1, keepdim=True)
    return u, dict(x=x, pre=pre, h=h, inv_a=inv_a, preb=preb, inv_b=inv_b)


def _net_forward(layers, x, nonlin, learn_thresh, eps, deltas=None):
    """f_theta0(x) and every block's activations (engine.py:161-175)."""
    s = len(layers) ** -0.5
    ctxs = []
    for l, layer in enumerate(layers):
        u, c = _net_block(layer, x, nonlin, learn_thresh, eps, None if deltas is None else deltas[l])
        ctxs.append(c)
        x = x + s * u
    return x, ctxs


def _net_scales(c, nonlin):
    """Per-branch column scales of dh/d(raw pre-activation) (engine.py:198-212)."""
    if nonlin == "swiglu":
        return [F.silu(c["preb"]) * c["inv_a"], c["pre"] * activation_grad("silu", c["preb"]) * c["inv_b"]]
    return [activation_grad(nonlin, c["pre"]) * c["inv_a"]]


def _net_write(layers, k, v, nonlin, learn_thresh, eps, iters):
    """LA1 / LA2 streams, iteration-major (engine.py:215-340)."""
    L = len(layers)
    s = L ** -0.5

    def solve(ctxs, r):
        diag = 0.0
        for (W1, W2, Wg), c in zip(layers, ctxs):
            s2 = sum(t * t for t in _net_scales(c, nonlin))
            diag = diag + (c["h"] * c["h"]).sum(-1, keepdim=True) + \
                (c["x"] * c["x"]).sum(-1, keepdim=True) * torch.einsum("hdm,bhtm->bhtd", W2 * W2, s2)
        return r / (diag / L + eps)

    def payloads(ctxs, lam):
        out = []
        for (W1, W2, Wg), c in zip(layers, ctxs):
            u2 = torch.einsum("hdm,bhtd->bhtm", W2, lam)
            out.append(s * torch.cat([t * u2 for t in _net_scales(c, nonlin)], dim=-1))
        return out

    o, ctxs = _net_forward(layers, k, nonlin, learn_thresh, eps)
    lam = solve(ctxs, v - o)
    gs = payloads(ctxs, lam)
    la1 = [(c["x"], g) for c, g in zip(ctxs, gs)]
    la2 = [(c["h"], s * lam) for c in ctxs]
    if iters == 2:
        deltas = [(c["x"], c["h"], s * lam, g) for c, g in zip(ctxs, gs)]
        o2, ctxs2 = _net_forward(layers, k, nonlin, learn_thresh, eps, deltas)
        lam2 = solve(ctxs2, v - o2)
        la1 += [(c["x"], g) for c, g in zip(ctxs2, payloads(ctxs2, lam2))]
        la2 += [(c["h"], s * lam2) for c in ctxs2]
    return la1, la2


def gn_core_net(q, k, v, layers, *, nonlin: str, learn_thresh: bool, read_norm: bool, read_norm_w1: bool,
                write_iters: int = 1, log_alphas=None, etas=None, mode: str = "fast", eps: float = 1e-6,
                chunk: int = 512, scan_fn=None):
    """GN mixer core of a net of any depth; ``layers`` = [(W1, W2, Wg)] per
    block (effective weights; Wg the swiglu gate [H,m,d] or the threshold
    [H,m,1])."""
    from .mixer import blend_outputs, view_terms
    if scan_fn is None:
        scan_fn = lambda qq, kk, vv, rets: scan.linattn_chunk_views(qq, kk, vv, rets, chunk)
    L = len(layers)
    s = L ** -0.5
    m = layers[0][1].shape[-1]
    la1, la2 = _net_write(layers, k, v, nonlin, learn_thresh, eps, write_iters)
    J = 0 if log_alphas is None else log_alphas.shape[0]
    retentions = tuple([None] + [log_alphas[j] for j in range(J)])

    def read(view, query, keys, vals, unit):
        if unit:
            vals = torch.cat([vals, vals.new_ones(*vals.shape[:3], 1)], dim=-1)
        return _combine(scan_fn(query, keys, vals, retentions), view)

    outs = []
    for view in view_terms(mode, J):
        x = q
        for l, (W1, W2, Wg) in enumerate(layers):
            a = torch.einsum("hmd,bhtd->bhtm", W1, x)
            b = torch.einsum("hmd,bhtd->bhtm", Wg, x) if nonlin == "swiglu" else None
            if read_norm_w1:
                h0 = activation("relu2", _net_features(a, None, Wg, "relu2", learn_thresh, eps)[0])
                c = read(view, h0, la2[l][0], la1[l][1], True)
                a = a + c[..., :m] / (c[..., -1:] + eps)
            else:
                for it in range(write_iters):
                    keys, vals = la1[it * L + l]
                    c = read(view, x, keys, vals, False)
                    a = a + c[..., :m]
                    if b is not None:
                        b = b + c[..., m:]
            h = _net_features(a, b, Wg, nonlin, learn_thresh, eps)[1]
            if read_norm:
                c = read(view, h, la2[l][0], la2[l][1], True)
                mem = c[..., :-1] / (c[..., -1:] + eps)
            else:
                mem = sum(read(view, h, la2[it * L + l][0], la2[it * L + l][1], False) for it in range(write_iters))
            x = x + s * (torch.einsum("hdm,bhtm->bhtd", W2, h) + mem)
        outs.append(x)
    base_out = None
    if J and mode == "stale":
        # the zero-memory read: every scan empty, so the net itself at q
        base_out = _net_forward(layers, q, nonlin, learn_thresh, eps)[0]
    return blend_outputs(outs, base_out, mode, etas) if J else outs[0]
