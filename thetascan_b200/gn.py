"""Gauss--Newton (GN) fast-weight family on the B200 path.

One memory block (depth 1) with one Jacobian step, as the reference runs
``family="gn"`` (src/thetascan/config.py:745-756).  Per token, in f32 with
autograd:

  write (engine.py:161-340)  a = W1 k, pre = rmsnorm(a) [- tau], h = sigma(pre),
                             o = k + W2 h, r = v - o,
                             lambda = r / (||h||^2 + ||k||^2 (W2^2)(s^2) + eps),
                             s = sigma'(pre) / rms(a),
                             g = sigma'(pre) (W2^T lambda) / rms(a);
  read (engine.py:455-528)   stage 1: pre_v = W1 q + [g-stream read of the view],
                             stage 2: h_v = sigma(rmsnorm(pre_v) [- tau]),
                             y_v = q + W2 h_v + [lambda-stream read of the view].

Every read over the sequence -- the T-long part -- runs on the sm_100a
multi-view scan kernels (``ts_b200_scan_fwd/bwd``) with bf16 streams, f32
states and f32 reads: stage 1 once for all views (one score tile per view
set), stage 2 once per view because each view's query differs
(engine.py:355-361).  The read normalizations follow the reference:
``both_feature_mass`` reads [g | 1] with the positive slow features
h0 = relu2(rmsnorm(W1 q) [- tau]) against keys h and normalizes both stages
by their mass column; ``w2_feature_mass`` reads g with q against k
unnormalized and normalizes stage 2; ``none`` normalizes neither.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from .scan import scan_views_f32


class _tf32:
    """TF32 tensor-core GEMMs for f32 matmuls inside the block (10-bit
    mantissa operands, f32 accumulation), restoring the caller's setting."""

    def __enter__(self):
        self.saved = torch.backends.cuda.matmul.allow_tf32
        torch.backends.cuda.matmul.allow_tf32 = True

    def __exit__(self, *exc):
        torch.backends.cuda.matmul.allow_tf32 = self.saved


class _PerToken(torch.autograd.Function):
    """``fn(*tensors)`` with TF32 GEMMs in the forward and in the backward,
    which recomputes ``fn`` under autograd (the per-token GN math is cheap next
    to its f32 SIMT GEMMs, and recomputation keeps nothing but the inputs)."""

    @staticmethod
    def forward(ctx, fn, *tensors):
        ctx.fn = fn
        ctx.save_for_backward(*tensors)
        with _tf32(), torch.no_grad():
            out = fn(*tensors)
        ctx.single = torch.is_tensor(out)
        return out

    @staticmethod
    def backward(ctx, *grads):
        inputs = [t.detach().requires_grad_(t.requires_grad) for t in ctx.saved_tensors]
        with _tf32():
            with torch.enable_grad():
                out = ctx.fn(*inputs)
            outs = [out] if ctx.single else list(out)
            pairs = [(o, g) for o, g in zip(outs, grads) if g is not None and o.requires_grad]
            wanted = [t for t in inputs if t.requires_grad]
            # the gradient GEMMs (the projections' weight gradients above all)
            # run inside the TF32 setting too
            got = torch.autograd.grad([o for o, _ in pairs], wanted, [g for _, g in pairs], allow_unused=True) \
                if pairs and wanted else [None] * len(wanted)
        it = iter(got)
        return (None, *[next(it) if t.requires_grad else None for t in inputs])


def per_token(fn, *tensors):
    """Run the per-token block ``fn`` on TF32 tensor cores (see _PerToken)."""
    return _PerToken.apply(fn, *tensors)


def per_token_f32(fn, *tensors):
    """The same block in full f32: the write's solve and the features, whose
    gradients (the log-retention one above all, a long sum over tokens) move
    by ~2% when their operands are rounded to TF32."""
    return fn(*tensors)


class _HeadMap(torch.autograd.Function):
    """``y[b,h,t] = W[h] x[b,h,t]`` for ``W [H,o,i]``, ``x [B,H,T,i]``, f32.

    The weight gradient sums over all B*T tokens of a head; as one GEMM per
    head (what an einsum's backward does) that is a handful of output tiles
    with a 10^5-long reduction, so few SMs work.  Here the token axis is cut
    into chunks that become batch entries (a view of the contiguous input),
    the per-chunk products run in parallel, and their sum is taken after."""

    @staticmethod
    def forward(ctx, W, x):
        ctx.save_for_backward(W, x)
        return torch.matmul(x, W.transpose(-1, -2).unsqueeze(0))

    @staticmethod
    def backward(ctx, gy):
        W, x = ctx.saved_tensors
        gW = gx = None
        if ctx.needs_input_grad[1]:
            gx = torch.matmul(gy, W.unsqueeze(0))
        if ctx.needs_input_grad[0]:
            B, H, T, i = x.shape
            o = gy.shape[-1]
            xc, gc = x.contiguous(), gy.contiguous()
            S = 1
            while T % (2 * S) == 0 and T // (2 * S) >= 512 and B * H * S < 512:
                S *= 2
            part = torch.bmm(gc.view(B * H * S, T // S, o).transpose(1, 2), xc.view(B * H * S, T // S, i))
            gW = part.view(B, H, S, o, i).sum(dim=(0, 2))
        return gW, gx


def head_map(W, x):
    """Per-head linear map ``y[b,h,t] = W[h] x[b,h,t]`` (see _HeadMap)."""
    return _HeadMap.apply(W, x)


def _activation(nonlin, pre):
    if nonlin == "relu2":
        r = F.relu(pre)
        return r * r
    if nonlin == "silu":
        return F.silu(pre)
    if nonlin == "tanh":
        return torch.tanh(pre)
    raise NotImplementedError(f"b200 GN: nonlinearity {nonlin!r} is not built")


def _activation_grad(nonlin, pre):
    if nonlin == "relu2":
        return 2.0 * F.relu(pre)
    if nonlin == "silu":
        s = torch.sigmoid(pre)
        return s * (1 + pre * (1 - s))
    if nonlin == "tanh":
        # sigma'(pre) = 1 - tanh(pre)^2, the table's (act, dact(pre, h)) pattern
        h = torch.tanh(pre)
        return 1.0 - h * h
    raise NotImplementedError(f"b200 GN: nonlinearity {nonlin!r} is not built")


def _rmsnorm(a, eps):
    """``a * rsqrt(mean(a^2) + eps)`` and the factor (reference norms.py:5-8)."""
    inv = torch.rsqrt(a.square().mean(-1, keepdim=True) + eps)
    return a * inv, inv


def _thresholded(pre, tau):
    return pre if tau is None else pre - tau[..., 0].unsqueeze(0).unsqueeze(2).to(pre.dtype)


def _views(mode, J):
    """Retention slots of each view: slot 0 the plain sum, 1+j branch j (its
    decayed scan for a fast bank, its stale scan for a stale bank)."""
    if J and mode not in ("fast", "stale"):
        raise ValueError(f"b200 GN: unknown bank mode {mode!r}")
    return [0] + [1 + j for j in range(J)]


def _piece_width(n_retentions, Dk):
    """Payload columns (unit column included) one scan call takes within the
    tensor-memory and shared-memory budget of its tile kernels."""
    if n_retentions >= 4:
        return 96
    if n_retentions == 3 or Dk > 128:
        return 128
    return 144


def _scan(query, keys, payload, append_unit, retentions, stale=None):
    """f32 reads of the multi-view scan kernels (bf16 streams, f32 gradients
    back).  The scan is linear in the payload, so a payload wider than one
    call takes is read in column pieces (the mass column rides on the last)."""
    width = payload.shape[-1]
    step = _piece_width(len(retentions), query.shape[-1]) - 1
    if width + (1 if append_unit else 0) <= step + 1:
        return scan_views_f32(query, keys, payload, append_unit, stale, retentions)
    parts = [[] for _ in retentions]
    for start in range(0, width, step):
        piece = payload[..., start:start + step]
        last = start + step >= width
        for i, read in enumerate(scan_views_f32(query, keys, piece, append_unit and last, stale, retentions)):
            parts[i].append(read)
    return tuple(torch.cat(p, dim=-1) for p in parts)


def gn_write(k, v, W1, W2, tau, nonlin, eps):
    """(h, g, lambda) of every token, f32 (reference engine.py:161-340, depth 1)."""
    a = head_map(W1, k)
    pre, inv = _rmsnorm(a, eps)
    pre = _thresholded(pre, tau)
    h = _activation(nonlin, pre)
    o = k + head_map(W2, h)
    r = v - o
    dsig = _activation_grad(nonlin, pre)
    s = dsig * inv
    rowsq = head_map(W2 * W2, s * s)
    diag = h.square().sum(-1, keepdim=True) + k.square().sum(-1, keepdim=True) * rowsq
    lam = r / (diag + eps)
    g = dsig * head_map(W2.transpose(1, 2), lam) * inv
    return h, g, lam


def gn_core(q, k, v, W1, W2, tau=None, *, nonlin="relu2", read_norm=True, read_norm_w1=True, log_alphas=None,
            etas=None, mode="fast", eps=1e-6):
    """GN mixer core ``[B,H,T,d]`` f32 from bf16 ``q, k, v`` after RoPE / L2 norm.

    ``W1 [H,m,d]``, ``W2 [H,d,m]`` effective weights, ``tau [H,m,1]`` the learned
    threshold of ``relu2_threshold`` (or None), ``log_alphas``/``etas``
    ``[J,H]`` for a fast bank."""
    for x in (q, k, v):
        if not x.is_cuda:
            raise RuntimeError("b200 backend requires CUDA tensors")
    m, d = W1.shape[1], q.shape[-1]
    qf, kf, vf = q.float(), k.float(), v.float()
    W1f, W2f = W1.float(), W2.float()
    tauf = None if tau is None else tau.float()
    extra = () if tauf is None else (tauf,)

    def write(kk, vv, w1, w2, *t):
        return gn_write(kk, vv, w1, w2, t[0] if t else None, nonlin, eps)

    h_k, g, lam = per_token_f32(write, kf, vf, W1f, W2f, *extra)
    J = 0 if log_alphas is None else log_alphas.shape[0]
    las = [None] + [log_alphas[j].float() for j in range(J)]
    slots = _views(mode, J)
    stale = [False] + [mode == "stale"] * J
    flags = stale if any(stale) else None

    def query_pre(qq, w1, *t):
        a = head_map(w1, qq)
        return a, _activation("relu2", _thresholded(_rmsnorm(a, eps)[0], t[0] if t else None))

    a_q, h0 = per_token_f32(query_pre, qf, W1f, *extra)
    # stage 1, shared by all views: the correction of the hidden preactivation
    if read_norm_w1:
        reads = _scan(h0, h_k, g, True, las, flags)
        pres = [a_q + reads[s][..., :m] / (reads[s][..., m:] + eps) for s in slots]
    else:
        reads = _scan(q, k, g, False, las, flags)
        pres = [a_q + reads[s] for s in slots]

    def features(pre, w2, *t):
        hq = _activation(nonlin, _thresholded(_rmsnorm(pre, eps)[0], t[0] if t else None))
        return hq, head_map(w2, hq)

    # stage 2, one query per view
    outs = []
    for s, pre in zip(slots, pres):
        hq, base = per_token_f32(features, pre, W2f, *extra)
        c = _scan(hq, h_k, lam, bool(read_norm), [las[s]], [True] if stale[s] else None)[0]
        mem = c[..., :d] / (c[..., d:] + eps) if read_norm else c
        outs.append(qf + base + mem)
    y = outs[0]
    if J and mode == "stale":
        # y - sum_j eta_j (y_stale_j - y_base), y_base the zero-memory read
        # (pre = W1 q, no memory term; block.py:697-718)
        y_base = qf + per_token_f32(features, a_q, W2f, *extra)[1]
        for j in range(J):
            y = y - etas[j].float().view(1, -1, 1, 1) * (outs[1 + j] - y_base)
        return y
    for j in range(J):
        y = y + etas[j].float().view(1, -1, 1, 1) * (outs[1 + j] - outs[0])
    return y
