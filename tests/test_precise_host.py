"""The float32 path's per-token math (thetascan_b200.precise) against the
oracle's restatement of the reference feature maps, on the CPU in float64
(the module's functions are device-agnostic PyTorch; only its scans need a
GPU).  Bit-for-bit agreement is not expected -- both are restatements of
kernel_features.py -- but float64 agreement to 1e-12 pins the formulas."""
from __future__ import annotations

import math

import pytest
import torch

from oracle import features as ofeatures
from oracle import mixer as omixer
from thetascan_b200.kernel import KernelSpec
from thetascan_b200 import precise


def _inputs(H=2, P=16, d=32, T=40, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(1, H, T, d, generator=g, dtype=torch.float64)
    W1 = torch.randn(H, P, d, generator=g, dtype=torch.float64) / math.sqrt(d)
    return x, W1, g


@pytest.mark.parametrize("controls", [False, True])
def test_relu2_features_match_oracle(controls):
    x, W1, g = _inputs()
    ctl = {}
    spec_o = {"kind": "relu2_ridge"}
    if controls:
        ctl["threshold"] = torch.randn(2, generator=g, dtype=torch.float64) * 0.1
        ctl["score_bias"] = torch.randn(2, 16, generator=g, dtype=torch.float64) * 0.2
        spec_o.update(relu2_threshold=ctl["threshold"], score_bias=ctl["score_bias"])
    got = precise.features(x, W1, KernelSpec(kind="relu2_ridge"), ctl)
    want = omixer.featurize(x, W1, spec_o, 1e-6)
    assert torch.allclose(got, want, rtol=1e-12, atol=1e-14)


@pytest.mark.parametrize("gain", ["fixed", "head", "feature"])
def test_softmax_features_match_oracle(gain):
    x, W1, g = _inputs()
    ctl, spec_o = {}, {"kind": "softmax_partition"}
    if gain == "head":
        ctl["gain"] = 4.0 + 8.0 * torch.rand(2, generator=g, dtype=torch.float64)
    elif gain == "feature":
        ctl["gain"] = 4.0 + 8.0 * torch.rand(2, 16, generator=g, dtype=torch.float64)
        ctl["score_bias"] = torch.randn(2, 16, generator=g, dtype=torch.float64) * 0.2
        spec_o["score_bias"] = ctl["score_bias"]
    spec_o["gain"] = ctl.get("gain", 8.0)
    got = precise.features(x, W1, KernelSpec(kind="softmax_partition"), ctl)
    want = omixer.featurize(x, W1, spec_o, 1e-6)
    assert torch.allclose(got, want, rtol=1e-12, atol=1e-14)


@pytest.mark.parametrize("basis", [8, 16])
def test_bspline_features_match_oracle(basis):
    x, W1, g = _inputs(P=8)
    scale = 0.5 + torch.rand(2, generator=g, dtype=torch.float64)
    got = precise.features(x, W1, KernelSpec(kind="projected_bspline", basis=basis), {"spline_scale": scale})
    want = omixer.featurize(x, W1, {"kind": "projected_bspline", "n_basis": basis, "scale": scale}, 1e-6)
    assert torch.allclose(got, want, rtol=1e-12, atol=1e-14)


def test_bspline_partition_matches_oracle_at_the_knots():
    """Coordinates on, just below and outside the knots, where the half-open
    spans and the clamp decide (kernel_features.py:138-205)."""
    bound, nb = 3.0, 16
    knots = ofeatures.open_uniform_knots(nb, 3, bound)
    c = torch.cat([knots, knots - 1e-9, torch.tensor([-5.0, 5.0, 0.0], dtype=torch.float64)])
    got = precise._bspline_partition(c, nb, bound)
    want = ofeatures.bspline_basis(c, n_basis=nb, degree=3, bound=bound)
    assert torch.allclose(got, want, rtol=1e-12, atol=1e-14)
