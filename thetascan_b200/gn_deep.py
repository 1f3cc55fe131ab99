"""GN memory nets beyond one relu2 / silu / tanh block: depth > 1 and swiglu.

The row kernels of :mod:`thetascan_b200.gn` run a GN net of depth 1 with an
elementwise activation.  This module runs every other GN net the reference
accepts -- any depth, the two-branch swiglu activation, one or two Jacobian
steps, all three read normalisations and every temporal view -- with the
sequence reads on the float32 multi-view scan kernels (custom op
``thetascan_b200::scan_views_fwd`` with float32 streams: f32 operands, states,
reads and gradients on the CUDA cores) and the per-token maps as float32
PyTorch under autograd.  Deep and swiglu nets amplify the rounding of their
scan operands: with bf16 operands the retention gradient of a swiglu net
with two Jacobian steps moved by 1-6% of its largest entry under rounding
perturbations alone, so these nets keep their streams in float32 (and their
per-token maps run in float32 under PyTorch's default matmul precision:
``torch.backends.cuda.matmul.allow_tf32`` left off).

Reference (src/thetascan/_core/ops/engine.py): the write is
``_forward_theta0`` / ``_block_forward`` (:117-175, residual
``x_{l+1} = x_l + u_l / sqrt(L)``), ``_lambda_solve`` (:215-255, the
Jacobi diagonal summed over the layers), ``_g_from_lambda`` (:180-195,
swiglu's payload ``[g_a | g_b]`` for both branches) and ``write_streams``
(:260-340, per layer ``LA1 = (x_l, g_l)``, ``LA2 = (h_l, lambda / sqrt(L))``;
the second Jacobian step re-runs the net with each token's own write
applied); the read is ``dual_read_views`` (:345-544): per layer, the hidden
correction scanned from LA1 (two-stage normalised for
``both_feature_mass``), the activation of the corrected pre-activation,
``W2 h`` plus the LA2 read, and views that share a query only until their
corrections differ (after the first layer every view runs alone).
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from . import scan as _scan
from .gn import _views
from .seqpar import sharded_reads

_ACTS = ("relu2", "silu", "tanh", "swiglu")


def _hm(W, x):
    """Per-head linear map ``y[b,h,t] = W[h] x[b,h,t]``."""
    return torch.matmul(x, W.transpose(-1, -2).unsqueeze(0))


def _rms(a, eps):
    """RMS normalisation and its scale ``1/rms`` (modules/norms.py:5-8)."""
    inv = torch.rsqrt(a.pow(2).mean(-1, keepdim=True) + eps)
    return a * inv, inv


def _dsilu(p):
    s = torch.sigmoid(p)
    return s * (1 + p * (1 - s))


def _act(nonlin, p):
    if nonlin == "relu2":
        r = F.relu(p)
        return r * r
    if nonlin == "silu":
        return F.silu(p)
    return torch.tanh(p)


def _dact(nonlin, p, h):
    if nonlin == "relu2":
        return 2.0 * F.relu(p)
    if nonlin == "silu":
        return _dsilu(p)
    return 1.0 - h * h


class _Block:
    """One block's activations at a token: input ``x``, normalised
    pre-activation ``pre`` (threshold applied), activation ``h``, ``1/rms``
    of the pre-activation ``inv_a``; swiglu adds its gate branch ``preb``
    and ``inv_b``."""

    __slots__ = ("x", "pre", "h", "inv_a", "preb", "inv_b")

    def __init__(self, x, pre, h, inv_a, preb=None, inv_b=None):
        self.x, self.pre, self.h, self.inv_a, self.preb, self.inv_b = x, pre, h, inv_a, preb, inv_b


class _Net:
    """The GN memory net: its layers ``(W1, W2, Wg)`` (``Wg`` the swiglu
    gate ``[H,m,d]`` or the learned threshold ``[H,m,1]``), activation and
    epsilon."""

    def __init__(self, layers, nonlin, thresholded, eps):
        self.layers, self.nonlin, self.eps = layers, nonlin, float(eps)
        self.thresholded = bool(thresholded)
        self.L = len(layers)
        self.s = 1.0 / math.sqrt(self.L)
        self.m = int(layers[0][1].shape[-1])

    def _threshold(self, pre, Wg):
        if not self.thresholded:
            return pre
        return pre - Wg[..., 0].unsqueeze(0).unsqueeze(2)

    def features(self, a, b, Wg):
        """Activation of a pre-activation (and swiglu's gate pre-activation)."""
        pre, inv_a = _rms(a, self.eps)
        if self.nonlin == "swiglu":
            preb, inv_b = _rms(b, self.eps)
            return pre, F.silu(preb) * pre, inv_a, preb, inv_b
        pre = self._threshold(pre, Wg)
        return pre, _act(self.nonlin, pre), inv_a, None, None

    def block(self, l, x, delta=None):
        """``u = W2 h(W1 x)`` of layer ``l`` and its activations; ``delta``
        applies a token's own first-step write (engine.py:117-158)."""
        W1, W2, Wg = self.layers[l]
        a = _hm(W1, x)
        b = _hm(Wg, x) if self.nonlin == "swiglu" else None
        if delta is not None:
            x0, h0, lam_hat, g = delta
            xx = (x0 * x).sum(-1, keepdim=True)
            a = a + g[..., :self.m] * xx
            if b is not None:
                b = b + g[..., self.m:] * xx
        pre, h, inv_a, preb, inv_b = self.features(a, b, Wg)
        u = _hm(W2, h)
        if delta is not None:
            u = u + lam_hat * (h0 * h).sum(-1, keepdim=True)
        return u, _Block(x, pre, h, inv_a, preb, inv_b)

    def forward0(self, x, deltas=None):
        """The net at its slow weights, ``f_theta0(x)``, and every block's
        activations (engine.py:161-175)."""
        blocks = []
        for l in range(self.L):
            u, blk = self.block(l, x, None if deltas is None else deltas[l])
            blocks.append(blk)
            x = x + self.s * u
        return x, blocks

    def _scales(self, blk):
        """Column scales ``s`` of ``Q = W2 diag(s)``, the Jacobian of one
        block's output in its raw pre-activation(s)."""
        if self.nonlin == "swiglu":
            return (F.silu(blk.preb) * blk.inv_a, blk.pre * _dsilu(blk.preb) * blk.inv_b)
        return (_dact(self.nonlin, blk.pre, blk.h) * blk.inv_a,)

    def solve(self, blocks, r):
        """Jacobi-preconditioned lambda (engine.py:215-255)."""
        diag = None
        for (W1, W2, Wg), blk in zip(self.layers, blocks):
            s2 = sum(c * c for c in self._scales(blk))
            term = (blk.h * blk.h).sum(-1, keepdim=True) + \
                (blk.x * blk.x).sum(-1, keepdim=True) * _hm(W2 * W2, s2)
            diag = term if diag is None else diag + term
        return r / (diag / self.L + self.eps)

    def payload(self, l, blk, lam):
        """``g = s * diag(scales) W2^T lambda`` of layer ``l``
        (engine.py:180-195; swiglu: ``[g_a | g_b]``)."""
        u2 = _hm(self.layers[l][1].transpose(1, 2), lam)
        return self.s * torch.cat([c * u2 for c in self._scales(blk)], dim=-1)

    def write(self, k, v, steps):
        """LA1 and LA2 streams, iteration-major (engine.py:260-340)."""
        o, blocks = self.forward0(k)
        lam = self.solve(blocks, v - o)
        la1 = [(blk.x, self.payload(l, blk, lam)) for l, blk in enumerate(blocks)]
        la2 = [(blk.h, self.s * lam) for blk in blocks]
        if steps == 2:
            deltas = [(blk.x, blk.h, self.s * lam, la1[l][1]) for l, blk in enumerate(blocks)]
            o2, blocks2 = self.forward0(k, deltas)
            lam2 = self.solve(blocks2, v - o2)
            la1 += [(blk.x, self.payload(l, blk, lam2)) for l, blk in enumerate(blocks2)]
            la2 += [(blk.h, self.s * lam2) for blk in blocks2]
        return la1, la2


def _pieces(width, unit, dk):
    """``(start, stop, unit)`` payload pieces within the float32 scan
    kernels' shared-memory budget (payload plus unit column: 240 columns for
    keys up to 128 wide, 120 beyond); the unit column rides the last piece."""
    step = (240 if dk <= 128 else 120) - 1
    if width + int(unit) <= step + 1:
        return [(0, width, unit)]
    return [(s, min(width, s + step), unit and min(width, s + step) >= width) for s in range(0, width, step)]


def _reads(query, keys, payload, unit, retentions, stale, shard=None):
    """Reads of one stream set through the views ``retentions`` (f32
    ``[B,H,T,W(+1)]`` each) on the float32 scan kernels, the payload cut into
    pieces within their budgets; on a sequence shard each piece enters with
    the earlier shards' state (:func:`thetascan_b200.seqpar.sharded_reads`)."""
    parts = [[] for _ in retentions]
    for start, stop, u in _pieces(int(payload.shape[-1]), unit, int(query.shape[-1])):
        piece = payload[..., start:stop].contiguous()
        if shard is None:
            outs = _scan.linattn_views(query, keys, piece, tuple(retentions), append_unit=bool(u),
                                       stale=tuple(stale))
        else:
            outs = sharded_reads(shard, _scan.linattn_views, query, keys, piece, tuple(retentions),
                                 append_unit=bool(u), stale=tuple(stale))
        for i, o in enumerate(outs):
            parts[i].append(o)
    return [p[0] if len(p) == 1 else torch.cat(p, dim=-1) for p in parts]


def _read(net, q, la1, la2, retentions, stale, read_norm, read_norm_w1, steps, shard=None):
    """Every view's read ``f_theta_t(q_t)`` (engine.py:345-544)."""
    L, m, eps = net.L, net.m, net.eps
    V = len(retentions)
    xs = [q] * V
    for l, (W1, W2, Wg) in enumerate(net.layers):
        # the first layer shares its query across the views; from the second
        # on, every view has its own corrected activations
        groups = [list(range(V))] if l == 0 else [[i] for i in range(V)]
        new = [None] * V
        for idx in groups:
            x = xs[idx[0]]
            rets, flags = [retentions[i] for i in idx], [stale[i] for i in idx]
            a = _hm(W1, x)
            b = _hm(Wg, x) if net.nonlin == "swiglu" else None
            if read_norm_w1:
                # two-stage read: positive relu2 features of the uncorrected
                # pre-activation address [g | 1] (engine.py:475-506)
                pre0 = net._threshold(_rms(a, eps)[0], Wg)
                h0 = _act("relu2", pre0)
                corr = _reads(h0, la2[l][0], la1[l][1], True, rets, flags, shard)
                pres = [a + c[..., :m] / (c[..., m:m + 1] + eps) for c in corr]
                bs = [b] * len(idx)
            else:
                pres, bs = [a] * len(idx), [b] * len(idx)
                for it in range(steps):
                    keys, vals = la1[it * L + l]
                    corr = _reads(x, keys, vals, False, rets, flags, shard)
                    pres = [p + c[..., :m] for p, c in zip(pres, corr)]
                    if b is not None:
                        bs = [bb + c[..., m:] for bb, c in zip(bs, corr)]
            for i, pre, bb in zip(idx, pres, bs):
                h = net.features(pre, bb, Wg)[1]
                base = _hm(W2, h)
                if read_norm:
                    c = _reads(h, la2[l][0], la2[l][1], True, [retentions[i]], [stale[i]], shard)[0]
                    mem = c[..., :-1] / (c[..., -1:] + eps)
                else:
                    mem = None
                    for it in range(steps):
                        keys, vals = la2[it * L + l]
                        c = _reads(h, keys, vals, False, [retentions[i]], [stale[i]], shard)[0]
                        mem = c if mem is None else mem + c
                new[i] = x + net.s * (base + mem)
        xs = new
    return xs


def gn_deep(q, k, v, layers, *, nonlin="relu2", thresholded=False, read_norm=False, read_norm_w1=False,
            log_alphas=None, etas=None, mode="fast", eps=1e-6, steps=1, shard=None):
    """GN mixer core ``[B,H,T,d]`` f32 of a net of any depth.

    ``q, k, v`` after RoPE / L2 norm; ``layers`` the per-layer effective
    weights ``(W1 [H,m,d], W2 [H,d,m], Wg)``, ``Wg`` the swiglu gate
    ``[H,m,d]``, the learned threshold ``[H,m,1]`` (``thresholded``) or None;
    ``nonlin`` relu2 / silu / tanh / swiglu; ``log_alphas`` / ``etas``
    ``[J,H]`` a temporal bank (``mode`` fast or stale); ``steps`` the
    Jacobian steps of the write; ``shard`` (a
    :class:`thetascan_b200.seqpar.SeqShard`) makes ``q, k, v`` one contiguous
    slice of longer sequences, every read entering with the earlier slices'
    state (one exchange per read).  Differentiable in every tensor argument."""
    for x in (q, k, v):
        if not x.is_cuda:
            raise RuntimeError("b200 backend requires CUDA tensors")
    if nonlin not in _ACTS:
        raise NotImplementedError(f"b200 GN: nonlinearity {nonlin!r} is not built")
    if steps not in (1, 2):
        raise ValueError("GNConfig.jacobian_steps must be 1 or 2")
    if (read_norm or read_norm_w1) and (steps != 1 or nonlin not in ("relu2",)):
        raise ValueError("GN feature-mass normalization requires relu2 features and jacobian_steps=1")
    J = 0 if log_alphas is None else int(log_alphas.shape[0])
    if J:
        _views(mode, J)
    return _core(q, k, v, layers, nonlin, thresholded, read_norm, read_norm_w1, log_alphas, etas, mode, eps,
                 steps, shard)


def _core(q, k, v, layers, nonlin, thresholded, read_norm, read_norm_w1, log_alphas, etas, mode, eps, steps,
          shard=None):
    """The GN core after the argument checks: write, reads of every view and
    the bank blend."""
    J = 0 if log_alphas is None else int(log_alphas.shape[0])
    net = _Net([(W1.float(), W2.float(), None if Wg is None else Wg.float()) for W1, W2, Wg in layers],
               nonlin, thresholded, eps)
    q, k, v = q.float(), k.float(), v.float()
    la1, la2 = net.write(k, v, steps)
    retentions = [None] + [log_alphas[j].float() for j in range(J)]
    stale = [False] + [mode == "stale"] * J
    ys = _read(net, q, la1, la2, retentions, stale, bool(read_norm), bool(read_norm_w1), steps, shard)
    y = ys[0]
    if J and mode == "stale":
        # y - sum_j eta_j (y_stale_j - y_base); y_base reads an empty memory,
        # which is the net itself at q (block.py:697-718)
        y_base = net.forward0(q)[0]
        for j in range(J):
            y = y - etas[j].float().view(1, -1, 1, 1) * (ys[1 + j] - y_base)
    elif J:
        for j in range(J):
            y = y + etas[j].float().view(1, -1, 1, 1) * (ys[1 + j] - ys[0])
    return y
