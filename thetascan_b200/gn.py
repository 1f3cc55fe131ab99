"""Gauss--Newton (GN) fast-weight family on the B200 path.

One memory block (depth 1) with one Jacobian step, as the reference runs
``family="gn"`` (src/thetascan/config.py:745-756).  Per token and head:

  write (engine.py:161-340)  a = W1 k, pre = rmsnorm(a) [- tau], h = sigma(pre),
                             o = k + W2 h, r = v - o,
                             lambda = r / (||h||^2 + ||k||^2 (W2^2)(s^2) + eps),
                             s = sigma'(pre) / rms(a),
                             g = sigma'(pre) (W2^T lambda) / rms(a);
  read (engine.py:455-528)   stage 1: pre_v = W1 q + [g-stream read of the view],
                             stage 2: h_v = sigma(rmsnorm(pre_v) [- tau]),
                             y_v = q + W2 h_v + [lambda-stream read of the view].

The core is one custom op (``thetascan_b200::gn_core_fwd`` with its
backward ``gn_core_bwd``): the nonlinear row maps run on the GN row kernels
(``ts_b200_gn_rows``: normalisation, activation and its derivatives, the
damped solve, the read normalisations, forward and backward, one HBM pass
each), the per-head linear maps (W1, W2, W2^T, W2 o W2 over all tokens of a
head) are float32 cuBLAS GEMMs, and every read over the sequence runs on
the sm_100a multi-view scan kernels with bf16 streams, f32 states and f32
reads: stage 1 once for all views (one score tile per view set), stage 2
once per view because each view's query differs (engine.py:355-361).  The
read normalizations follow the reference: ``both_feature_mass`` reads
[g | 1] with the positive slow features h0 = relu2(rmsnorm(W1 q) [- tau])
against keys h and normalizes both stages by their mass column;
``w2_feature_mass`` reads g with q against k unnormalized and normalizes
stage 2; ``none`` normalizes neither.  The backward is written out by hand
(no recomputation under autograd).
"""
from __future__ import annotations

import ctypes

import torch
import torch.nn.functional as F

from . import _lib
from .scan import _scan_bwd_impl, _scan_fwd_impl, _stream


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


class _Tf32Linear(torch.autograd.Function):
    """``F.linear`` whose forward and backward GEMMs both run on TF32 tensor
    cores (the autograd engine runs a backward outside the caller's TF32
    setting); saves its input and weight, no recomputation."""

    @staticmethod
    def forward(ctx, x, w, b):
        ctx.save_for_backward(x, w)
        ctx.has_bias = b is not None
        with _tf32():
            return F.linear(x, w, b)

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        with _tf32():
            dx = dy @ w if ctx.needs_input_grad[0] else None
            dw = dy.reshape(-1, dy.shape[-1]).t() @ x.reshape(-1, x.shape[-1]) if ctx.needs_input_grad[1] else None
        db = dy.reshape(-1, dy.shape[-1]).sum(0) if ctx.has_bias and ctx.needs_input_grad[2] else None
        return dx, dw, db


def tf32_linear(x, w, b=None):
    """``F.linear(x, w, b)`` with TF32 GEMMs forward and backward."""
    return _Tf32Linear.apply(x, w, b)


def per_token(fn, *tensors):
    """Run the per-token block ``fn`` on TF32 tensor cores (see _PerToken)."""
    return _PerToken.apply(fn, *tensors)


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


# --------------------------------------------------------------------------- GN core on the row kernels

_NONLIN = {"relu2": _lib.TS_GN_RELU2, "silu": _lib.TS_GN_SILU, "tanh": _lib.TS_GN_TANH}


class _Run:
    """One GN core evaluation: its shape, the row-kernel launcher and the
    allocator.  With ``fake`` set (the custom op's fake implementation)
    nothing is launched and only the shapes of the results are formed, so
    that the real and fake outputs come from one code path."""

    def __init__(self, q, m, tau, nonlin, eps, fake):
        if nonlin not in _NONLIN:
            raise NotImplementedError(f"b200 GN: nonlinearity {nonlin!r} is not built")
        self.B, self.H, self.T, self.d = (int(x) for x in q.shape)
        self.m, self.nl, self.eps, self.fake = int(m), _NONLIN[nonlin], float(eps), fake
        self.like = q
        self.tau = None if tau is None else tau[..., 0].float().contiguous()   # [H, m]
        self.tf32 = False   # per-head maps and weight-gradient products on TF32 (the core sets it)

    def new(self, width, zero=False, dtype=torch.float32):
        shape = (self.B, self.H, self.T) + ((width,) if width else ())
        f = torch.zeros if zero else torch.empty
        return f(shape, dtype=dtype, device=self.like.device)

    def new_bf16(self, width):
        return self.new(width, dtype=torch.bfloat16)

    def rows(self, stage, ins, outs, flags=0, dtau=None, bf16=None):
        """One row stage; ``bf16`` receives a bf16 copy of ``outs[0]`` (the
        scans' operand), and ``outs[0]`` may then be None for the stages
        whose first output feeds only the scans."""
        if self.fake:
            return
        a = _lib.GnRowsArgs()
        a.batch, a.heads, a.tokens, a.d, a.m = self.B, self.H, self.T, self.d, self.m
        a.nonlinearity, a.eps, a.stage, a.flags = self.nl, self.eps, stage, flags
        a.tau = None if self.tau is None else self.tau.data_ptr()
        a.dtau = None if dtau is None else dtau.data_ptr()
        for i, x in enumerate(ins):
            a.inputs[i] = None if x is None else x.data_ptr()
        for i, x in enumerate(outs):
            a.outputs[i] = None if x is None else x.data_ptr()
        a.out_bf16 = None if bf16 is None else bf16.data_ptr()
        _lib.check(_lib.load().ts_b200_gn_rows(ctypes.byref(a), _stream()))

    # ----------------------------------------------------------- scans

    def scan_fwd(self, query, keys, payload, unit, rets, stale):
        """Reads of every retention (f32, ``[B,H,T,W(+1)]``) and the state the
        backward needs: one scan call per payload piece (see _piece_width)."""
        pieces, reads = [], [[] for _ in rets]
        for start, stop, u in _scan_pieces(payload.shape[-1], unit, len(rets), query.shape[-1]):
            piece = payload[..., start:stop]
            if self.fake:
                from .ops import _scan_workspace_nbytes
                outs = self.like.new_empty(len(rets), self.B, self.H, self.T, stop - start + int(u),
                                           dtype=torch.float32)
                nbytes = _scan_workspace_nbytes(self.B, self.H, self.T, int(query.shape[-1]), stop - start, int(u),
                                                [r is not None for r in rets], stale, False)
                ws = self.like.new_empty(nbytes, dtype=torch.uint8)
            else:
                outs, ws = _scan_fwd_impl(query, keys, piece.contiguous(), rets, int(u), list(stale), True)
            pieces.append((start, stop, u, outs, ws))
            for i in range(len(rets)):
                reads[i].append(outs[i])
        return [r[0] if len(r) == 1 else torch.cat(r, dim=-1) for r in reads], pieces

    def scan_bwd(self, douts, query, keys, payload, pieces, rets, stale):
        """Gradients of query, keys, payload and the ``[R,H]`` log-retentions
        from the reads' gradients ``douts`` (one per retention)."""
        dq = dk = None
        dla = torch.zeros(len(rets), self.H, dtype=torch.float32, device=self.like.device)
        dp = []
        for start, stop, u, outs, ws in pieces:
            w = stop - start + int(u)
            g = [d_[..., start:start + w] for d_ in douts]
            if self.fake:
                pq, pk = torch.empty_like(query, dtype=torch.float32), torch.empty_like(keys, dtype=torch.float32)
                pv = self.new(stop - start)
            else:
                pq, pk, pv, pla, _ = _scan_bwd_impl(g, query, keys, payload[..., start:stop].contiguous(), rets,
                                                    outs, ws, int(u), list(stale), True)
                dla += pla
            dq = pq if dq is None else dq + pq
            dk = pk if dk is None else dk + pk
            dp.append(pv)
        return dq, dk, dp[0] if len(dp) == 1 else torch.cat(dp, dim=-1), dla


def _hm(W, x, tf32=False):
    """Per-head linear map ``y[b,h,t] = W[h] x[b,h,t]`` (batched GEMM); with
    ``tf32`` on TF32 tensor cores (10-bit operand mantissas, f32
    accumulation), else in f32 whatever the global TF32 setting."""
    saved = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = bool(tf32)
    try:
        return torch.matmul(x, W.transpose(-1, -2).unsqueeze(0))
    finally:
        torch.backends.cuda.matmul.allow_tf32 = saved


def _hm_acc(base, W, x, tf32=False):
    """``base + W[h] x[b,h,t]`` per head, the sum formed by the GEMM itself
    (beta = 1: no separate elementwise pass over ``[B,H,T,o]``)."""
    B, H, T, i = x.shape
    o = W.shape[1]
    Wt = W.transpose(-1, -2).unsqueeze(0).expand(B, H, i, o).reshape(B * H, i, o)
    saved = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = bool(tf32)
    try:
        out = torch.baddbmm(base.contiguous().view(B * H, T, o), x.contiguous().view(B * H, T, i), Wt)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = saved
    return out.view(B, H, T, o)


def _hm_wgrad(gy, x, tf32=False):
    """``sum_{b,t} gy[b,h,t] x[b,h,t]^T`` per head, ``[H,o,i]``: the token axis
    cut into chunks that run as parallel batched products, summed after in
    f32.  With ``tf32`` the products run on TF32 tensor cores (the GN core's
    setting: a weight gradient sums ~10^5 products, so the operands' 10-bit
    rounding averages out to ~1e-4 of it)."""
    B, H, T, i = x.shape
    o = gy.shape[-1]
    S = 1
    while T % (2 * S) == 0 and T // (2 * S) >= 512 and B * H * S < 512:
        S *= 2
    saved = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = bool(tf32)
    try:
        part = torch.bmm(gy.contiguous().view(B * H * S, T // S, o).transpose(1, 2),
                         x.contiguous().view(B * H * S, T // S, i))
    finally:
        torch.backends.cuda.matmul.allow_tf32 = saved
    return part.view(B, H, S, o, i).sum(dim=(0, 2))


def _gn_forward(q, k, v, W1, W2, tau, log_alphas, etas, nonlin, read_norm, read_norm_w1, mode, eps, fake,
                steps=1):
    """The GN core: ``y`` and the tensors its backward reads (a flat list, in
    the order _gn_backward takes them)."""
    B, H, T, d = q.shape
    m = W1.shape[1]
    run = _Run(q, m, tau, nonlin, eps, fake)
    run.tf32 = True
    W1, W2 = W1.float().contiguous(), W2.float().contiguous()
    J = 0 if log_alphas is None else int(log_alphas.shape[0])
    las = [None] + [log_alphas[j].float() for j in range(J)]
    stale = [False] + [mode == "stale"] * J
    a_k, h_k, s2, hh, kk, O, RS, lam, U, g, h_kb, lamb, g32 = _write_forward(run, k, v, W1, W2, bf16=True,
                                                                           g32=steps == 2)
    two = None
    if steps == 2:
        # the second Jacobian step (engine.py:323-339) and its streams
        two = _write2_forward(run, k, v, W2, a_k, h_k, kk, lam, g32)
        g = torch.cat([g, two["g2b"]], dim=-1)   # both g payloads in one stage-1 scan
    # stage 1, shared by all views (engine.py:475-500)
    a_q = _hm(W1, q, run.tf32)
    if read_norm_w1:
        h0 = run.new_bf16(m)
        run.rows(_lib.TS_GN_QUERY_PRE, [a_q], [None], bf16=h0)
        R1, st1 = run.scan_fwd(h0, h_kb, g, True, las, stale)
    else:
        h0 = q.new_empty(0)
        R1, st1 = run.scan_fwd(q, k, g, False, las, stale)
    saved = [a_k, h_k, h_kb, s2, hh, kk, O, RS, lam, lamb, U, g, a_q, h0]
    if two is not None:
        saved += [g32] + [two[n] for n in _WRITE2_SAVED]
        # the two g streams' reads add up (same query and keys)
        R1 = [r[..., :m] + r[..., m:] for r in R1]
    saved += [x for piece in st1 for x in piece[3:]]
    ys = []
    # stage 2, one query per view (engine.py:500-528)
    for s in range(J + 1):
        hq, hqb = run.new(m), run.new_bf16(m)
        run.rows(_lib.TS_GN_FEATURES, [a_q, R1[s]], [hq], flags=int(read_norm_w1), bf16=hqb)
        base = _hm(W2, hq, run.tf32)
        (C,), st2 = run.scan_fwd(hqb, h_kb, lamb, bool(read_norm), [las[s]], [stale[s]])
        saved += [hq, hqb] + [x for piece in st2 for x in piece[3:]]
        if two is not None:
            # the second step's lambda stream against its own keys h2
            (C2,), st2b = run.scan_fwd(hqb, two["h2b"], two["lam2b"], False, [las[s]], [stale[s]])
            C = C + C2
            saved += [x for piece in st2b for x in piece[3:]]
        y = run.new(d)
        run.rows(_lib.TS_GN_OUT, [q, base, C], [y], flags=int(bool(read_norm)))
        ys.append(y)
    y = ys[0]
    if J and mode == "stale":
        # y - sum_j eta_j (y_stale_j - y_base), y_base the zero-memory read
        # (pre = W1 q, no memory term; block.py:697-718)
        hb = run.new(m)
        run.rows(_lib.TS_GN_FEATURES, [a_q, None], [hb])
        y_base = q + _hm(W2, hb, run.tf32)
        for j in range(J):
            y = y - etas[j].float().view(1, -1, 1, 1) * (ys[1 + j] - y_base)
        saved += ys + [y_base]
    elif J:
        for j in range(J):
            y = y + etas[j].float().view(1, -1, 1, 1) * (ys[1 + j] - ys[0])
        saved += ys
    return y, saved


def _take(saved, n):
    out, rest = saved[:n], saved[n:]
    return out, rest


def _gn_backward(dy, q, k, v, W1, W2, tau, log_alphas, etas, saved, nonlin, read_norm, read_norm_w1, mode, eps,
                 fake, steps=1):
    """Gradients of the GN core: q, k, v, W1, W2, tau, log_alphas, etas."""
    B, H, T, d = q.shape
    m = W1.shape[1]
    run = _Run(q, m, tau, nonlin, eps, fake)
    run.tf32 = True
    W1, W2 = W1.float().contiguous(), W2.float().contiguous()
    W2t = W2.transpose(1, 2)
    J = 0 if log_alphas is None else int(log_alphas.shape[0])
    las = [None] + [log_alphas[j].float() for j in range(J)]
    stale = [False] + [mode == "stale"] * J
    (a_k, h_k, h_kb, s2, hh, kk, O, RS, lam, lamb, U, g, a_q, h0), rest = _take(saved, 14)
    two = g32 = None
    if steps == 2:
        (g32,), rest = _take(rest, 1)
        vals, rest = _take(rest, len(_WRITE2_SAVED))
        two = dict(zip(_WRITE2_SAVED, vals))
    q1 = h0 if read_norm_w1 else q
    k1 = h_kb if read_norm_w1 else k
    w1 = m * steps   # stage-1 payload: the g stream of each step
    n1 = len(_scan_pieces(w1, bool(read_norm_w1), J + 1, q1.shape[-1]))
    flat1, rest = _take(rest, 2 * n1)
    st1 = _pieces(w1, bool(read_norm_w1), J + 1, q1.shape[-1], flat1)
    views = []
    for s in range(J + 1):
        (hq, hqb), rest = _take(rest, 2)
        n2 = len(_scan_pieces(d, bool(read_norm), 1, m))
        flat2, rest = _take(rest, 2 * n2)
        st2b = None
        if steps == 2:
            flat2b, rest = _take(rest, 2 * len(_scan_pieces(d, False, 1, m)))
            st2b = _pieces(d, False, 1, m, flat2b)
        views.append((hq, hqb, _pieces(d, bool(read_norm), 1, m, flat2), st2b))
    dy = dy.float().contiguous()
    # the view combination
    tau_grad = None if tau is None else torch.zeros(H, m, dtype=torch.float32, device=q.device)
    dla = torch.zeros(J + 1, H, dtype=torch.float32, device=q.device)
    deta = None if J == 0 else torch.zeros(J, H, dtype=torch.float32, device=q.device)
    # q enters every view and the zero-memory base with coefficients that sum
    # to one: its direct gradient is dy itself (added with the last product)
    dys = [dy]
    dy_base = None
    if J:
        ys, rest = _take(rest, J + 1)
        e = etas.float()
        if mode == "stale":
            (y_base,), rest = _take(rest, 1)
            dys = [dy] + [-e[j].view(1, -1, 1, 1) * dy for j in range(J)]
            dy_base = e.sum(0).view(1, -1, 1, 1) * dy
            for j in range(J):
                deta[j] = -(dy * (ys[1 + j] - y_base)).sum(dim=(0, 2, 3))
        else:
            dys = [(1.0 - e.sum(0)).view(1, -1, 1, 1) * dy] + [e[j].view(1, -1, 1, 1) * dy for j in range(J)]
            for j in range(J):
                deta[j] = (dy * (ys[1 + j] - ys[0])).sum(dim=(0, 2, 3))
    dW2 = torch.zeros_like(W2)
    dh_k = dlam = None
    da_q = run.new(m)
    R1 = [torch.cat([p[3][i] for p in st1], dim=-1) if len(st1) > 1 else st1[0][3][i] for i in range(J + 1)]
    if steps == 2:
        R1 = [r[..., :m] + r[..., m:] for r in R1]
        dh2 = run.new(m, zero=True)
        dlam2 = run.new(d, zero=True)
    dR1 = [run.new(R1[0].shape[-1]) for _ in range(J + 1)]
    for s, (hq, hqb, st2, st2b) in enumerate(views):
        C = st2[0][3][0] if len(st2) == 1 else torch.cat([p[3][0] for p in st2], dim=-1)
        if read_norm:
            dC = run.new(d + 1)
            run.rows(_lib.TS_GN_OUT_BWD, [dys[s], C], [dC], flags=1)
        else:
            dC = dys[s]
        dhq, dhk_s, dlam_s, dla_s = run.scan_bwd([dC], hqb, h_kb, lamb, st2, [las[s]], [stale[s]])
        dh_k = dhk_s if dh_k is None else dh_k + dhk_s
        dlam = dlam_s if dlam is None else dlam + dlam_s
        dla[s] += dla_s[0]
        if st2b is not None:
            dhq2, dh2_s, dlam2_s, dla2_s = run.scan_bwd([dC], hqb, two["h2b"], two["lam2b"], st2b, [las[s]],
                                                        [stale[s]])
            dhq = dhq + dhq2
            dh2 += dh2_s
            dlam2 += dlam2_s
            dla[s] += dla2_s[0]
        dhq = _hm_acc(dhq, W2t, dys[s], run.tf32)
        dW2 += _hm_wgrad(dys[s], hq, run.tf32)
        run.rows(_lib.TS_GN_FEATURES_BWD, [a_q, R1[s], dhq], [da_q, dR1[s]],
                 flags=int(read_norm_w1) | (2 if s else 0), dtau=tau_grad)
    if dy_base is not None:
        hb = run.new(m)
        run.rows(_lib.TS_GN_FEATURES, [a_q, None], [hb])
        dW2 += _hm_wgrad(dy_base, hb, run.tf32)
        run.rows(_lib.TS_GN_FEATURES_BWD, [a_q, None, _hm(W2t, dy_base, run.tf32)], [da_q, None], flags=2,
                 dtau=tau_grad)
    # stage 1
    if steps == 2:
        dR1 = [torch.cat([r, r], dim=-1) for r in dR1]
    dq1, dk1, dg, dla1 = run.scan_bwd(dR1, q1, k1, g, st1, las, stale)
    dla += dla1
    dk = None
    if read_norm_w1:
        dh_k += dk1
        run.rows(_lib.TS_GN_QUERY_PRE_BWD, [dq1, a_q], [da_q], flags=2, dtau=tau_grad)
        dq = _hm_acc(dy, W1.transpose(1, 2), da_q, run.tf32)
    else:
        dk = dk1
        dq = _hm_acc(dy + dq1, W1.transpose(1, 2), da_q, run.tf32)
    dW1 = _hm_wgrad(da_q, q, run.tf32)
    da_extra = None
    if steps == 2:
        dg, dg2 = dg[..., :m].contiguous(), dg[..., m:].contiguous()
        dk2, dv2, dW2_2, da_extra, dg_f, dh_f, dlam_f = _write2_backward(
            run, k, v, W2, two, h_k, lam, g32, kk, dh2, dg2, dlam2, tau_grad)
        dg = dg + dg_f
        dh_k += dh_f
        dlam += dlam_f
        dW2 += dW2_2
        dk = dk2 if dk is None else dk + dk2
    dk_w, dv, dW1_w, dW2_w = _write_backward(run, k, v, W1, W2, (a_k, h_k, s2, hh, kk, O, RS, lam, U),
                                             dh_k, dg, dlam, tau_grad, da_extra)
    if steps == 2:
        dv = dv + dv2
    dk = dk_w if dk is None else dk_w + dk
    return dq, dk, dv, dW1 + dW1_w, dW2 + dW2_w, tau_grad, dla[1:], deta


def _write_forward(run, k, v, W1, W2, bf16=False, g32=False):
    """The GN write (engine.py:161-340): ``a = W1 k`` and the row streams
    ``h, s2, hh, kk, O, RS, lam, U, g`` (h the keys, g and lam the payloads of
    the two read stages; the rest kept for the backward).  With ``bf16`` the
    row kernels also write the scans' bf16 operands: g in bf16 (and in f32
    with ``g32``), and ``(h_bf16, lam_bf16, g_f32 or None)`` follow the
    tuple."""
    m, d = run.m, run.d
    # The write's maps stay f32: the damped solve divides by them, and TF32
    # operands here moved the log-retention gradient by ~0.4% of its largest
    # entry (the read and backward maps run on TF32 without a visible shift).
    a_k = _hm(W1, k)
    h_k, s2, hh, kk = run.new(m), run.new(m), run.new(0), run.new(0)
    h_kb = run.new_bf16(m) if bf16 else None
    run.rows(_lib.TS_GN_WRITE_PRE, [a_k, k], [h_k, s2, hh, kk], bf16=h_kb)
    O, RS = _hm(W2, h_k), _hm(W2 * W2, s2)
    lam = run.new(d)
    lamb = run.new_bf16(d) if bf16 else None
    run.rows(_lib.TS_GN_WRITE_LAM, [v, k, O, RS, hh, kk], [lam], bf16=lamb)
    U = _hm(W2.transpose(1, 2), lam)
    if bf16:
        g, gf = run.new_bf16(m), (run.new(m) if g32 else None)
        run.rows(_lib.TS_GN_WRITE_G, [a_k, U], [gf], bf16=g)
        return a_k, h_k, s2, hh, kk, O, RS, lam, U, g, h_kb, lamb, gf
    g = run.new(m)
    run.rows(_lib.TS_GN_WRITE_G, [a_k, U], [g])
    return a_k, h_k, s2, hh, kk, O, RS, lam, U, g


_WRITE2_SAVED = ("a2", "h2", "h2b", "s2b", "hh2", "O2", "RS2", "lam2", "lam2b", "U2", "hd")


def _write2_forward(run, k, v, W2, a_k, h_k, kk, lam, g):
    """The second Jacobian step (``write_iters == 2``, engine.py:323-339):
    the block re-run at theta0 plus this token's first-step write
    (engine.py:117-158 with ``delta``): a2 = a + g |k|^2, h2 = sigma(rms(a2) -
    tau), O2 = W2 h2 + lam (h . h2), then the same damped solve for lam2 and
    g2 = sigma'(p2) (W2^T lam2) / rms(a2).  The read adds the (k, g2) and
    (h2, lam2) streams to the first step's."""
    m, d = run.m, run.d
    a2 = a_k + g * kk.unsqueeze(-1)
    h2, s2b, hh2, kk2 = run.new(m), run.new(m), run.new(0), run.new(0)
    h2b = run.new_bf16(m)
    run.rows(_lib.TS_GN_WRITE_PRE, [a2, k], [h2, s2b, hh2, kk2], bf16=h2b)
    hd = (h_k * h2).sum(-1, keepdim=True)
    O2 = _hm(W2, h2) + lam * hd
    RS2 = _hm(W2 * W2, s2b)
    lam2, lam2b = run.new(d), run.new_bf16(d)
    run.rows(_lib.TS_GN_WRITE_LAM, [v, k, O2, RS2, hh2, kk], [lam2], bf16=lam2b)
    U2 = _hm(W2.transpose(1, 2), lam2)
    g2b = run.new_bf16(m)
    run.rows(_lib.TS_GN_WRITE_G, [a2, U2], [None], bf16=g2b)
    return dict(a2=a2, h2=h2, h2b=h2b, s2b=s2b, hh2=hh2, O2=O2, RS2=RS2, lam2=lam2, lam2b=lam2b, U2=U2, hd=hd,
                g2b=g2b)


def _write2_backward(run, k, v, W2, two, h_k, lam, g, kk, dh2, dg2, dlam2, dtau):
    """Backward of the second step from the gradients of its streams (h2,
    g2, lam2): returns (d k, d v, d W2, d a2) of its own terms and the
    gradients it hands to the first step's g, h and lam."""
    m, d = run.m, run.d
    W2t = W2.transpose(1, 2)
    du2 = run.new(m)
    run.rows(_lib.TS_GN_WRITE_G_BWD, [dg2, two["a2"]], [du2])
    dlam2W = _hm(W2, du2, run.tf32)
    dr2, drowsq2, dk2, dhh2 = run.new(d), run.new(d), run.new(d), run.new(0)
    run.rows(_lib.TS_GN_WRITE_LAM_BWD, [dlam2, dlam2W, v, k, two["O2"], two["RS2"], two["hh2"], kk],
             [dr2, drowsq2, dk2, dhh2])
    h2 = two["h2"]
    tf = run.tf32
    dW2 = (_hm_wgrad(two["lam2"], du2, tf) - _hm_wgrad(dr2, h2, tf)
           + 2.0 * W2 * _hm_wgrad(drowsq2, two["s2b"], tf))
    # O2 = W2 h2 + lam (h . h2), and r2 = v - k - O2
    dhd = -(dr2 * lam).sum(-1, keepdim=True)
    dlam_first = -dr2 * two["hd"]
    dh_first = dhd * h2
    ds2 = _hm((W2 * W2).transpose(1, 2), drowsq2, run.tf32)
    dhO2 = _hm(W2t, dr2, run.tf32)
    da2 = run.new(m)
    run.rows(_lib.TS_GN_WRITE_PRE_BWD, [dh2 + dhd * h_k, dhO2, ds2, dhh2, dg2, two["U2"], two["a2"]], [da2],
             dtau=dtau)
    # a2 = a + g |k|^2
    dg_first = da2 * kk.unsqueeze(-1)
    dk2 = dk2 + 2.0 * (da2 * g).sum(-1, keepdim=True) * k
    return dk2, dr2, dW2, da2, dg_first, dh_first, dlam_first


def _write_backward(run, k, v, W1, W2, streams, dh, dg, dlam, dtau, da_extra=None):
    """Gradients of k, v, W1, W2 (and tau into ``dtau``) of the write from
    those of its outputs h, g, lam (and ``da_extra``, a gradient of a = W1 k
    from elsewhere)."""
    a_k, h_k, s2, hh, kk, O, RS, lam, U = streams
    m, d = run.m, run.d
    W2t = W2.transpose(1, 2)
    du = run.new(m)
    run.rows(_lib.TS_GN_WRITE_G_BWD, [dg, a_k], [du])
    dlamW = _hm(W2, du, run.tf32)
    dv, drowsq, dk_w, dhh = run.new(d), run.new(d), run.new(d), run.new(0)
    run.rows(_lib.TS_GN_WRITE_LAM_BWD, [dlam, dlamW, v, k, O, RS, hh, kk], [dv, drowsq, dk_w, dhh])
    tf = run.tf32
    dW2 = _hm_wgrad(lam, du, tf) - _hm_wgrad(dv, h_k, tf) + 2.0 * W2 * _hm_wgrad(drowsq, s2, tf)
    ds2 = _hm((W2 * W2).transpose(1, 2), drowsq, run.tf32)
    dhO = _hm(W2t, dv, run.tf32)
    da_k = run.new(m)
    run.rows(_lib.TS_GN_WRITE_PRE_BWD, [dh, dhO, ds2, dhh, dg, U, a_k], [da_k], dtau=dtau)
    if da_extra is not None:
        da_k = da_k + da_extra
    dk = _hm_acc(dk_w, W1.transpose(1, 2), da_k, run.tf32)
    return dk, dv, _hm_wgrad(da_k, k, run.tf32), dW2


def _scan_pieces(width, unit, n_retentions, dk):
    step = _piece_width(n_retentions, dk) - 1
    if width + int(unit) <= step + 1:
        return [(0, width, unit)]
    return [(s, min(width, s + step), unit and min(width, s + step) >= width) for s in range(0, width, step)]


def _pieces(width, unit, n_retentions, dk, flat):
    """The scan state of the payload pieces from the flat saved list."""
    return [(a, b, u, flat[2 * i], flat[2 * i + 1]) for i, (a, b, u) in enumerate(_scan_pieces(width, unit,
                                                                                                 n_retentions, dk))]


def gn_core(q, k, v, W1, W2, tau=None, *, nonlin="relu2", read_norm=True, read_norm_w1=True, log_alphas=None,
            etas=None, mode="fast", eps=1e-6, steps=1):
    """GN mixer core ``[B,H,T,d]`` f32 from ``q, k, v`` after RoPE / L2 norm.

    ``W1 [H,m,d]``, ``W2 [H,d,m]`` effective weights, ``tau [H,m,1]`` the learned
    threshold of ``relu2_threshold`` (or None), ``log_alphas``/``etas``
    ``[J,H]`` for a bank, ``steps`` the Jacobian steps of the write (2: the
    reference's ``write_iters == 2``, unnormalised reads only).  Runs as the
    ``thetascan_b200::gn_core`` custom op
    (the row kernels of ``ts_b200_gn_rows``, cuBLAS for the per-head maps,
    the multi-view scan kernels for the reads)."""
    for x in (q, k, v):
        if not x.is_cuda:
            raise RuntimeError("b200 backend requires CUDA tensors")
    if nonlin not in _NONLIN:
        raise NotImplementedError(f"b200 GN: nonlinearity {nonlin!r} is not built")
    if steps not in (1, 2):
        raise NotImplementedError(f"b200 GN: {steps} Jacobian steps")
    if steps == 2 and (read_norm or read_norm_w1):
        raise ValueError("GN feature-mass normalization requires jacobian_steps=1")
    J = 0 if log_alphas is None else log_alphas.shape[0]
    if J:
        _views(mode, J)
    from . import ops  # noqa: F401  (registers the operators)
    y, _ = torch.ops.thetascan_b200.gn_core_fwd(
        q.float().contiguous(), k.float().contiguous(), v.float().contiguous(), W1, W2, tau,
        log_alphas, etas, nonlin, bool(read_norm), bool(read_norm_w1), mode if J else "sum", float(eps), int(steps))
    return y
