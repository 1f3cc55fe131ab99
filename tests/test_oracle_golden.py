"""Pin the CPU oracle to fixtures recorded from the reference package.

Each fixture under ``tests/golden/`` was produced by the reference ThetaScan
itself (``tests/golden/make_golden.py``); nothing here imports the reference.
"""
from __future__ import annotations

import os

import pytest
import torch

from oracle import features, mixer, scan

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _load(name):
    return torch.load(os.path.join(GOLDEN, name), weights_only=False)


def _close(got, want, tol=1e-9):
    torch.testing.assert_close(got, want, rtol=tol, atol=tol)


# ----------------------------------------------------------------- scan level

@pytest.mark.parametrize("index", [0, 1, 2])
def test_chunk_oracle_matches_reference_outputs_and_grads(index):
    case = _load("scan_cases.pt")["cases"][index]
    q, k, v, ret = case["q"], case["k"], case["v"], case["retention"]
    leaves = [x.clone().requires_grad_(True) for x in (q, k, v)]
    r = None if ret is None else ret.clone().requires_grad_(True)
    if r is not None and r.ndim == 1:
        out = scan.linattn_chunk(*leaves, chunk=case["chunk"], log_alpha=r)
    else:
        out = scan.linattn_chunk(*leaves, r, chunk=case["chunk"])
    _close(out, case["out"])
    out.square().sum().backward()
    for got, want in zip([x.grad for x in leaves] + [None if r is None else r.grad], case["grads"]):
        if want is None:
            assert got is None
        else:
            _close(got, want, 1e-8)


@pytest.mark.parametrize("index", [0, 1, 2])
def test_naive_and_quad_oracles_match_reference_naive(index):
    case = _load("scan_cases.pt")["cases"][index]
    q, k, v, ret = case["q"], case["k"], case["v"], case["retention"]
    stream = scan._as_stream(ret, q)
    _close(scan.linattn_naive(q, k, v, stream), case["naive"])
    _close(scan.linattn_quad(q, k, v, stream), case["naive"])


def test_cumsum_and_multi_view_oracles_match_reference():
    data = _load("scan_cases.pt")
    q, k, v, la = data["views_inputs"]
    _close(scan.linattn_cumsum(q, k, v), data["cumsum_sum"])
    views = scan.linattn_chunk_views(q, k, v, (None, la, la * 3.0), chunk=16)
    for got, want in zip(views, data["views"]):
        _close(got, want)


def test_chunk_oracle_rejects_like_the_reference():
    q = torch.randn(1, 2, 9, 4, dtype=torch.float64)
    with pytest.raises(NotImplementedError):
        scan.linattn_chunk(q, q, q, -torch.rand_like(q))
    with pytest.raises(ValueError):
        scan.linattn_chunk(q, q, q, chunk=0)
    with pytest.raises(ValueError):
        scan.linattn_chunk(q, q, q, chunk=4, log_alpha=torch.zeros(3, dtype=torch.float64))


# ----------------------------------------------------------------- features

def test_feature_maps_match_reference():
    f = _load("feature_cases.pt")
    _close(features.relu2_ridge(f["pre"], threshold=f["thr"]), f["relu2"])
    _close(features.relu2_ridge(f["pre"], score_bias=f["bias"]), f["relu2_bias"])
    _close(features.relu2_ridge(-f["pre"].abs() - 1.0), f["relu2_dead"])
    _close(features.softmax_partition(f["pre"], gain=f["gain"], score_bias=f["bias"]), f["softmax"])
    _close(features.projected_bspline(f["spline_pre"], n_basis=8), f["bspline"])
    _close(features.projected_bspline(f["spline_pre"], n_basis=16), f["bspline16"])
    _close(features.bspline_basis(f["edge"], n_basis=8), f["bspline_edge"])


def test_bspline_partition_of_unity_and_support():
    """Known answer: each projection's basis sums to one with <= 4 nonzeros
    (reference tests/test_kernel_feature_maps.py:214-228)."""
    x = torch.linspace(-4.0, 4.0, 401, dtype=torch.float64)
    basis = features.bspline_basis(x, n_basis=16)
    _close(basis.sum(-1), torch.ones_like(x))
    assert int((basis > 0).sum(-1).max()) <= 4


# ----------------------------------------------------------------- mixer level

MIXER_CASES = ["softmax_bank_fast", "relu2_expanded_rope", "bspline_stale",
               "softmax_sum_feature_mass", "relu2_d64_ragged"]


def _core_cfg(case):
    c = dict(case["core"])
    c["read_norm"] = c["read_norm_mode"] if c.pop("read_norm") else "none"
    return c


@pytest.mark.parametrize("name", MIXER_CASES)
def test_mixer_oracle_matches_reference_forward_and_backward(name):
    case = _load("mixer_cases.pt")[name]
    dtype = case["x"].dtype
    params = {n: t.to(torch.float64).clone().requires_grad_(t.is_floating_point() and not n.startswith("_"))
              for n, t in case["params"].items()}
    x = case["x"].to(torch.float64).clone().requires_grad_(True)
    y = mixer.mixer_forward(params, _core_cfg(case), x)
    tol = 1e-9 if dtype == torch.float64 else 2e-6
    _close(y, case["y"].to(torch.float64), tol)
    (y * case["out_weight"].to(torch.float64)).sum().backward()
    _close(x.grad, case["x_grad"].to(torch.float64), tol)
    for n, g in case["grads"].items():
        _close(params[n].grad, g.to(torch.float64), tol)


def test_expansion_maps_match_reference_buffers():
    case = _load("mixer_cases.pt")["relu2_expanded_rope"]
    m, b = case["params"]["_expand_w1_0"].shape[1:]
    key = case["core"]["expansion_key"]
    u = mixer.row_map((1, m, b), key=key, role="w1-expand-layer-0")
    d = mixer.row_map((1, b, m), key=key, role="w2-expand-layer-0")
    assert torch.equal(u.to(torch.float64), case["params"]["_expand_w1_0"])
    assert torch.equal(d.to(torch.float64), case["params"]["_expand_w2_0"])


GN_CASES = ["gn_both_relu2_bank", "gn_both_threshold_expanded", "gn_w2_relu2_sum", "gn_none_silu_bank2",
            "gn_d64_ragged", "gn_d64_stale"]


@pytest.mark.parametrize("name", GN_CASES)
def test_gn_mixer_oracle_matches_reference_forward_and_backward(name):
    """The GN restatement (oracle/gn.py) against the reference GN mixer: output,
    input gradient and every parameter gradient."""
    case = _load("gn_cases.pt")[name]
    dtype = case["x"].dtype
    params = {n: t.to(torch.float64).clone().requires_grad_(t.is_floating_point() and not n.startswith("_"))
              for n, t in case["params"].items()}
    x = case["x"].to(torch.float64).clone().requires_grad_(True)
    cfg = dict(case["core"])
    y = mixer.mixer_forward(params, cfg, x)
    # The float32 fixture stores inputs rounded after the reference ran in
    # float64; the lambda solve's division amplifies that rounding to ~6e-6.
    tol = 1e-9 if dtype == torch.float64 else 2e-5
    _close(y, case["y"].to(torch.float64), tol)
    (y * case["out_weight"].to(torch.float64)).sum().backward()
    _close(x.grad, case["x_grad"].to(torch.float64), tol)
    for n, g in case["grads"].items():
        _close(params[n].grad, g.to(torch.float64), tol)


@pytest.mark.parametrize("file,name", [("gn_c3_cases.pt", "gn_c3_d128_T1024"),
                                       ("gn_tanh_cases.pt", "gn_tanh_d128_sum"),
                                       ("gn_tanh_cases.pt", "gn_tanh_d128_bank2")])
def test_gn_oracle_matches_reference_at_config3_width(file, name):
    """The GN restatement at config 3's widths (head_dim 128, m = 128): the
    relu2 two-stage read, and the tanh net with damping 1e-2 and the
    unnormalized read -- config 3 as the baseline states it, which the
    reference engine runs once its nonlinearity table holds tanh and its core
    epsilon is 1e-2 (tests/golden/make_golden.py, gn_tanh_cases)."""
    case = _load(file)[name]
    params = {n: t.to(torch.float64).clone().requires_grad_(t.is_floating_point() and not n.startswith("_"))
              for n, t in case["params"].items()}
    x = case["x"].to(torch.float64).clone().requires_grad_(True)
    y = mixer.mixer_forward(params, dict(case["core"]), x)
    # float32 fixtures of float64 runs: the stored inputs are rounded
    tol = 2e-5
    _close(y, case["y"].to(torch.float64), tol)
    (y * case["out_weight"].to(torch.float64)).sum().backward()
    _close(x.grad, case["x_grad"].to(torch.float64), tol)
    for n, g in case["grads"].items():
        _close(params[n].grad, g.to(torch.float64), tol)


@pytest.mark.parametrize("mode", ["relative_soft", "relative_st", "relative_st_blend"])
def test_relative_sparsity_matches_reference(mode):
    """The softmax partition's relative sparsity (kernel_features.py:43-113):
    the map and its gradients to the scores, the cutoff and the blend."""
    case = _load("sparse_cases.pt")["features"][mode]
    pre = case["pre"].clone().requires_grad_(True)
    rho = case["rho"].clone().requires_grad_(True)
    alpha = case["alpha"].clone().requires_grad_(True)
    phi = features.softmax_partition(pre, gain=case["gain"], score_bias=case["bias"], sparsity=mode, rho=rho,
                                     blend=alpha if mode == "relative_st_blend" else None)
    _close(phi, case["phi"])
    (phi * case["weight"]).sum().backward()
    _close(pre.grad, case["dpre"], 1e-8)
    _close(rho.grad, case["drho"], 1e-8)
    if mode == "relative_st_blend":
        _close(alpha.grad, case["dalpha"], 1e-8)


@pytest.mark.parametrize("name", ["softmax_relative_soft", "softmax_relative_st", "softmax_relative_st_blend"])
def test_sparse_mixer_oracle_matches_reference(name):
    """The oracle mixer with relative sparsity against the reference mixer
    (float32 fixtures: output, input gradient, every parameter gradient)."""
    case = _load("sparse_cases.pt")["mixers"][name]
    params = {n: t.to(torch.float64).clone().requires_grad_(t.is_floating_point() and not n.startswith("_"))
              for n, t in case["params"].items()}
    x = case["x"].to(torch.float64).clone().requires_grad_(True)
    y = mixer.mixer_forward(params, _core_cfg(case), x)

    def rel(got, want):   # the fixture is stored in float32: relative to its largest entry
        want = want.to(torch.float64)
        return float((got.detach() - want).abs().max() / want.abs().max())

    assert rel(y, case["y"]) < 1e-6
    (y * case["out_weight"].to(torch.float64)).sum().backward()
    assert rel(x.grad, case["x_grad"]) < 1e-6
    for n, g in case["grads"].items():
        assert rel(params[n].grad, g) < 1e-6, n


@pytest.mark.parametrize("file,name", [("gn_deep_cases.pt", n) for n in (
    "gn_swiglu_sum", "gn_swiglu_jac2_bank", "gn_depth2_both_bank", "gn_depth2_swiglu_stale",
    "gn_depth3_threshold_w2_expanded", "gn_depth2_silu_jac2_bank2")] + [
    ("gn_jac2_cases.pt", "gn_jac2_relu2_bank"), ("gn_jac2_cases.pt", "gn_jac2_threshold_sum")])
def test_gn_net_oracle_matches_reference(file, name):
    """The general GN net restatement (oracle/gn.py: depth > 1, swiglu, two
    Jacobian steps) against the reference GN mixer's fixtures: output, input
    gradient and every parameter gradient."""
    case = _load(file)[name]
    params = {n: t.to(torch.float64).clone().requires_grad_(t.is_floating_point() and not n.startswith("_"))
              for n, t in case["params"].items()}
    x = case["x"].to(torch.float64).clone().requires_grad_(True)
    y = mixer.mixer_forward(params, dict(case["core"]), x)
    (y * case["out_weight"].to(torch.float64)).sum().backward()

    # float32 fixtures of float64 runs: the stored inputs are rounded, which
    # these nets' solves amplify on small entries (up to 1e-3 of an entry,
    # 1.5e-6 of a quantity's largest); the bound is on the largest entry
    def rel(got, want):
        want = want.to(torch.float64)
        return float((got.detach() - want).abs().max() / want.abs().max())

    tol = 1e-5
    assert rel(y, case["y"]) < tol
    assert rel(x.grad, case["x_grad"]) < tol
    for n, g in case["grads"].items():
        assert rel(params[n].grad, g) < tol, n
