"""GPU numerics of the GN row kernels (``ts_b200_gn_rows``) against plain
PyTorch float64 references of the same maps, forward and backward.

The write (engine.py:161-340 of the reference: normalisation, threshold,
activation, the damped diagonal solve, g) runs through the package's own
orchestration (``gn._write_forward`` / ``gn._write_backward``: row kernels
plus float32 cuBLAS per-head maps); the read stages (the slow features h0,
the corrected features of a view, the mass-normalised output) call the row
kernels directly.  Inputs are float32; the references run in float64 on the
same values.  Bound: ``max|got - ref| / max|ref| <= 1e-5``.
"""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu
TOL = 1e-5


def rel_err(got, want):
    got = got.detach().to("cpu", torch.float64)
    want = want.detach().to("cpu", torch.float64)
    return float((got - want).abs().max() / want.abs().max().clamp_min(1e-30))


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda")


def _act(nl, x):
    if nl == "relu2":
        return torch.relu(x) ** 2
    if nl == "silu":
        return torch.nn.functional.silu(x)
    return torch.tanh(x)


def _dact(nl, x):
    if nl == "relu2":
        return 2.0 * torch.relu(x)
    if nl == "silu":
        s = torch.sigmoid(x)
        return s * (1 + x * (1 - s))
    return 1.0 - torch.tanh(x) ** 2


def _hm(W, x):
    return torch.einsum("hoi,bhti->bhto", W, x)


def _rms(a, eps):
    inv = torch.rsqrt(a.square().mean(-1, keepdim=True) + eps)
    return a * inv, inv


def _thr(p, tau):
    return p if tau is None else p - tau[..., 0].view(1, tau.shape[0], 1, -1)


def _write_ref(k, v, W1, W2, tau, nl, eps):
    a = _hm(W1, k)
    n, inv = _rms(a, eps)
    p = _thr(n, tau)
    h = _act(nl, p)
    ds = _dact(nl, p)
    r = v - k - _hm(W2, h)
    s = ds * inv
    diag = h.square().sum(-1, keepdim=True) + k.square().sum(-1, keepdim=True) * _hm(W2 * W2, s * s)
    lam = r / (diag + eps)
    g = ds * _hm(W2.transpose(1, 2), lam) * inv
    return h, g, lam


def _inputs(dev, B, H, T, d, m, threshold, seed):
    g = torch.Generator().manual_seed(seed)
    k = torch.nn.functional.normalize(torch.randn(B, H, T, d, generator=g), dim=-1)
    v = torch.randn(B, H, T, d, generator=g)
    W1 = torch.randn(H, m, d, generator=g) / d ** 0.5
    W2 = torch.randn(H, d, m, generator=g) * 0.05
    tau = (torch.rand(H, m, 1, generator=g) * 0.5) if threshold else None
    return [None if x is None else x.to(dev) for x in (k, v, W1, W2, tau)]


WIDTHS = [(2, 3, 70, 64, 128), (1, 2, 130, 128, 128), (1, 2, 65, 64, 256), (1, 1, 33, 48, 80)]


@pytest.mark.parametrize("eps", [1e-6, 1e-2])
@pytest.mark.parametrize("threshold", [False, True])
@pytest.mark.parametrize("nl", ["relu2", "silu", "tanh"])
@pytest.mark.parametrize("shape", WIDTHS)
def test_gn_write_rows_match_float64(dev, shape, nl, threshold, eps):
    from thetascan_b200 import _lib, gn
    B, H, T, d, m = shape
    k, v, W1, W2, tau = _inputs(dev, B, H, T, d, m, threshold, seed=d + m)
    run = gn._Run(k, m, tau, nl, eps, False)
    streams = gn._write_forward(run, k, v, W1, W2)
    h, lam, g = streams[1], streams[7], streams[9]
    leaves = [x.double().requires_grad_(True) for x in (k, v, W1, W2)]
    tl = None if tau is None else tau.double().requires_grad_(True)
    want = _write_ref(*leaves, tl, nl, eps)
    for got, w in zip((h, g, lam), want):
        assert rel_err(got, w) < TOL
    gen = torch.Generator().manual_seed(5)
    grads = [torch.randn(w.shape, generator=gen, dtype=torch.float64) for w in want]
    sum((w * gg.to(dev)).sum() for w, gg in zip(want, grads)).backward()
    dtau = None if tau is None else torch.zeros(H, m, device=dev)
    dk, dv, dW1, dW2 = gn._write_backward(run, k, v, W1, W2, streams[:9], *(gg.float().to(dev) for gg in grads),
                                          dtau)
    assert _lib.device_status(torch.cuda.current_stream().cuda_stream) == 0
    for name, got, leaf in zip(("k", "v", "W1", "W2"), (dk, dv, dW1, dW2), leaves):
        assert rel_err(got, leaf.grad) < TOL, name
    if tau is not None:
        assert rel_err(dtau, tl.grad[..., 0]) < TOL


def _rows(run, stage, ins, outs, flags=0, dtau=None):
    run.rows(stage, ins, outs, flags=flags, dtau=dtau)


@pytest.mark.parametrize("read", ["normalised", "plain", "none"])
@pytest.mark.parametrize("threshold", [False, True])
@pytest.mark.parametrize("nl", ["relu2", "silu", "tanh"])
def test_gn_read_feature_rows_match_float64(dev, nl, threshold, read):
    """pre = a_q + R[:m] / (R[m] + eps) (or + R, or a_q alone), hq =
    sigma(rms(pre) - tau): forward, d a_q (accumulated), dR and d tau."""
    from thetascan_b200 import _lib, gn
    B, H, T, d, m = 2, 3, 77, 64, 128
    eps = 1e-2
    gen = torch.Generator().manual_seed(11)
    a_q = torch.randn(B, H, T, m, generator=gen)
    width = m + 1 if read == "normalised" else m
    R = torch.randn(B, H, T, width, generator=gen)
    if read == "normalised":
        R[..., m] = R[..., m].abs() + 0.5
    tau = (torch.rand(H, m, 1, generator=gen) * 0.5) if threshold else None
    dhq = torch.randn(B, H, T, m, generator=gen)
    prior = torch.randn(B, H, T, m, generator=gen)
    a_q, R, dhq, prior = (x.to(dev) for x in (a_q, R, dhq, prior))
    tau = None if tau is None else tau.to(dev)
    run = gn._Run(a_q.new_empty(B, H, T, d), m, tau, nl, eps, False)
    Rk = None if read == "none" else R
    flags = int(read == "normalised")
    hq = run.new(m)
    _rows(run, _lib.TS_GN_FEATURES, [a_q, Rk], [hq], flags)
    da = prior.clone()
    dR = run.new(width)
    dtau = None if tau is None else torch.zeros(H, m, device=dev)
    _rows(run, _lib.TS_GN_FEATURES_BWD, [a_q, Rk, dhq], [da, dR if Rk is not None else None], flags | 2, dtau)
    al, Rl = a_q.double().requires_grad_(True), R.double().requires_grad_(True)
    tl = None if tau is None else tau.double().requires_grad_(True)
    if read == "normalised":
        pre = al + Rl[..., :m] / (Rl[..., m:] + eps)
    elif read == "plain":
        pre = al + Rl
    else:
        pre = al
    want = _act(nl, _thr(_rms(pre, eps)[0], tl))
    (want * dhq.double()).sum().backward()
    assert _lib.device_status(torch.cuda.current_stream().cuda_stream) == 0
    assert rel_err(hq, want) < TOL
    assert rel_err(da - prior, al.grad) < TOL
    if Rk is not None:
        assert rel_err(dR, Rl.grad) < TOL
    if tau is not None:
        assert rel_err(dtau, tl.grad[..., 0]) < TOL


@pytest.mark.parametrize("threshold", [False, True])
def test_gn_slow_query_features_match_float64(dev, threshold):
    """h0 = relu2(rms(a_q) - tau), the positive slow features of the
    two-stage read, and its gradient (accumulated into d a_q)."""
    from thetascan_b200 import _lib, gn
    B, H, T, m = 2, 2, 90, 256
    eps = 1e-6
    gen = torch.Generator().manual_seed(13)
    a_q, dh, prior = (torch.randn(B, H, T, m, generator=gen).to(dev) for _ in range(3))
    tau = (torch.rand(H, m, 1, generator=gen) * 0.5).to(dev) if threshold else None
    run = gn._Run(a_q.new_empty(B, H, T, 64), m, tau, "tanh", eps, False)
    h0 = run.new(m)
    _rows(run, _lib.TS_GN_QUERY_PRE, [a_q], [h0])
    da = prior.clone()
    dtau = None if tau is None else torch.zeros(H, m, device=dev)
    _rows(run, _lib.TS_GN_QUERY_PRE_BWD, [dh, a_q], [da], 2, dtau)
    al = a_q.double().requires_grad_(True)
    tl = None if tau is None else tau.double().requires_grad_(True)
    want = torch.relu(_thr(_rms(al, eps)[0], tl)) ** 2
    (want * dh.double()).sum().backward()
    assert rel_err(h0, want) < TOL
    assert rel_err(da - prior, al.grad) < TOL
    if tau is not None:
        assert rel_err(dtau, tl.grad[..., 0]) < TOL


@pytest.mark.parametrize("normalised", [True, False])
def test_gn_read_output_rows_match_float64(dev, normalised):
    """y = q + base + C[:d] / (C[d] + eps) (or + C) and dC."""
    from thetascan_b200 import _lib, gn
    B, H, T, d = 2, 3, 100, 128
    eps = 1e-2
    gen = torch.Generator().manual_seed(17)
    q, base, dy = (torch.randn(B, H, T, d, generator=gen).to(dev) for _ in range(3))
    C = torch.randn(B, H, T, d + int(normalised), generator=gen)
    if normalised:
        C[..., d] = C[..., d].abs() + 0.25
    C = C.to(dev)
    run = gn._Run(q, 64, None, "relu2", eps, False)
    y = run.new(d)
    _rows(run, _lib.TS_GN_OUT, [q, base, C], [y], int(normalised))
    Cl = C.double().requires_grad_(True)
    want = q.double() + base.double() + ((Cl[..., :d] / (Cl[..., d:] + eps)) if normalised else Cl)
    assert rel_err(y, want) < TOL
    if normalised:
        dC = run.new(d + 1)
        _rows(run, _lib.TS_GN_OUT_BWD, [dy, C], [dC], 1)
        (want * dy.double()).sum().backward()
        assert rel_err(dC, Cl.grad) < TOL


def test_gn_rows_errors(dev):
    import ctypes
    from thetascan_b200 import _lib
    lib = _lib.load()
    a = _lib.GnRowsArgs()
    a.batch, a.heads, a.tokens, a.d, a.m = 1, 1, 4, 8, 300
    a.stage = _lib.TS_GN_WRITE_PRE
    assert lib.ts_b200_gn_rows(ctypes.byref(a), None) == _lib.TS_ERR_NOT_IMPLEMENTED   # m > 256
    a.m = 8
    assert lib.ts_b200_gn_rows(ctypes.byref(a), None) == _lib.TS_ERR_VALUE             # missing rows
    a.stage = 99
    assert lib.ts_b200_gn_rows(ctypes.byref(a), None) == _lib.TS_ERR_VALUE
    a.stage, a.nonlinearity = _lib.TS_GN_WRITE_PRE, 7
    assert lib.ts_b200_gn_rows(ctypes.byref(a), None) == _lib.TS_ERR_NOT_IMPLEMENTED


@pytest.mark.parametrize("d,rot", [(128, 64), (64, 64), (96, 0), (256, 128)])
def test_gn_prep_matches_float64(dev, d, rot):
    """q, k, v of the GN mixer from its fused projection: the split, RoPE on
    the first ``rot`` channels and x / max(|x|, eps) of q and k (block.py:
    577-599), forward and backward, against float64 on the same values."""
    import thetascan_b200.ops  # noqa: F401
    from thetascan_b200.mixer import _rope_tables
    B, T, H = 2, 150, 3
    eps = 1e-2
    gen = torch.Generator().manual_seed(d + rot)
    qkv = torch.randn(B, T, 3 * H * d, generator=gen).to(dev)
    qkv[0, 3, :H * d] *= 1e-4                       # one q row below the norm floor
    if rot:
        cos, sin = _rope_tables(T, rot, 10000.0, str(dev))
    else:
        cos = sin = qkv.new_empty(0)
    leaf = qkv.clone().requires_grad_(True)
    q, k, v = torch.ops.thetascan_b200.gn_prep_fwd(leaf, cos, sin, rot, H, eps)
    grads = [torch.randn(B, H, T, d, generator=gen).to(dev) for _ in range(3)]
    sum((o * g_).sum() for o, g_ in zip((q, k, v), grads)).backward()

    ref = qkv.double().requires_grad_(True)
    rq, rk, rv = ref.view(B, T, 3, H, d).permute(2, 0, 3, 1, 4)

    def rope_l2(x):
        if rot:
            c, s = cos.double(), sin.double()
            e, o = x[..., 0:rot:2], x[..., 1:rot:2]
            x = torch.cat((torch.stack((e * c - o * s, e * s + o * c), -1).flatten(-2), x[..., rot:]), -1)
        return x / x.norm(dim=-1, keepdim=True).clamp_min(eps)

    want = (rope_l2(rq), rope_l2(rk), rv)
    sum((o * g_.double()).sum() for o, g_ in zip(want, grads)).backward()
    for got, w in zip((q, k, v), want):
        assert got.is_contiguous() and rel_err(got, w) < TOL
    assert rel_err(leaf.grad, ref.grad) < TOL


@pytest.mark.parametrize("threshold", [False, True])
@pytest.mark.parametrize("nl", ["relu2", "tanh"])
def test_gn_two_step_write_matches_float64(dev, nl, threshold):
    """Two Jacobian steps (engine.py:117-158 with the this-token delta,
    323-339): the second step's streams h2, g2, lam2 and the gradients of
    both steps' six streams with respect to k, v, W1, W2 and tau, against
    float64 autograd of the same maps."""
    from thetascan_b200 import _lib, gn
    B, H, T, d, m = 2, 2, 70, 64, 128
    eps = 1e-2
    k, v, W1, W2, tau = _inputs(dev, B, H, T, d, m, threshold, seed=7)
    run = gn._Run(k, m, tau, nl, eps, False)
    st = gn._write_forward(run, k, v, W1, W2, bf16=True, g32=True)
    a_k, h_k, kk, lam, g32 = st[0], st[1], st[4], st[7], st[12]
    two = gn._write2_forward(run, k, v, W2, a_k, h_k, kk, lam, g32)
    g2 = run.new(m)
    run.rows(_lib.TS_GN_WRITE_G, [two["a2"], two["U2"]], [g2])

    leaves = [x.double().requires_grad_(True) for x in (k, v, W1, W2)]
    tl = None if tau is None else tau.double().requires_grad_(True)
    kd, vd, W1d, W2d = leaves
    h, g, lm = _write_ref(kd, vd, W1d, W2d, tl, nl, eps)
    kkd = kd.square().sum(-1, keepdim=True)
    a2 = _hm(W1d, kd) + g * kkd
    n2, inv2 = _rms(a2, eps)
    p2 = _thr(n2, tl)
    h2, ds2 = _act(nl, p2), _dact(nl, p2)
    O2 = _hm(W2d, h2) + lm * (h * h2).sum(-1, keepdim=True)
    s2 = ds2 * inv2
    lam2 = (vd - kd - O2) / (h2.square().sum(-1, keepdim=True) + kkd * _hm(W2d * W2d, s2 * s2) + eps)
    g2d = ds2 * _hm(W2d.transpose(1, 2), lam2) * inv2
    want = (h, g, lm, h2, g2d, lam2)
    for got, w in zip((h_k, g32, lam, two["h2"], g2, two["lam2"]), want):
        assert rel_err(got, w) < TOL
    gen = torch.Generator().manual_seed(6)
    cot = [torch.randn(w.shape, generator=gen, dtype=torch.float64) for w in want]
    sum((w * c.to(dev)).sum() for w, c in zip(want, cot)).backward()
    dh, dg, dlam, dh2, dg2, dlam2 = (c.float().to(dev) for c in cot)
    dtau = None if tau is None else torch.zeros(H, m, device=dev)
    dk2, dv2, dW2_2, da2, dg_f, dh_f, dlam_f = gn._write2_backward(run, k, v, W2, two, h_k, lam, g32, kk, dh2,
                                                                   dg2, dlam2, dtau)
    dk1, dv1, dW1, dW2_1 = gn._write_backward(run, k, v, W1, W2, st[:9], dh + dh_f, dg + dg_f, dlam + dlam_f,
                                              dtau, da2)
    assert _lib.device_status(torch.cuda.current_stream().cuda_stream) == 0
    for name, got, leaf in zip(("k", "v", "W1", "W2"), (dk1 + dk2, dv1 + dv2, dW1, dW2_1 + dW2_2), leaves):
        assert rel_err(got, leaf.grad) < TOL, name
    if tau is not None:
        assert rel_err(dtau, tl.grad[..., 0]) < TOL
