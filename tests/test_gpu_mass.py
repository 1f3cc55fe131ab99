"""GPU parity of the per-feature mass kernels of the feature-mass read.

``ts_b200_mass_query_fwd/bwd`` against the float64 oracle's
``causal_prefix_sum`` / ``ema_cumsum`` (and their difference for the stale
view), the reference's ``mass_cum`` (interface.py:58-107, 216-230, 278-279):
q_scaled = phi_q / (mass + eps), and the gradients of phi_q, phi_k and the
log-retention.  Tolerance: bf16 output rounding (2e-2 of the largest value).
"""
from __future__ import annotations

import math

import pytest
import torch

from oracle import scan as oscan

pytestmark = pytest.mark.gpu
BF16_TOL = 2e-2


def rel_err(got, want):
    got = got.detach().to("cpu", torch.float64)
    want = want.detach().to("cpu", torch.float64)
    return float((got - want).abs().max() / want.abs().max().clamp_min(1e-30))


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda")


def _oracle(phi_k, phi_q, la, kind, eps):
    if kind == "sum":
        mass = oscan.causal_prefix_sum(phi_k)
    elif kind == "fast":
        mass = oscan.ema_cumsum(phi_k, la, 64)
    else:
        mass = oscan.causal_prefix_sum(phi_k) - oscan.ema_cumsum(phi_k, la, 64)
    return phi_q / (mass + eps)


@pytest.mark.parametrize("kind", ["sum", "fast", "stale"])
@pytest.mark.parametrize("B,H,T,m", [(1, 2, 37, 16), (2, 3, 700, 128), (1, 2, 300, 256)])
def test_mass_query_matches_oracle(dev, kind, B, H, T, m):
    from thetascan_b200.kernel import _MassQuery
    g = torch.Generator().manual_seed(T + m)
    # positive features, as the feature maps produce
    phi_k = torch.rand(B, H, T, m, generator=g).to(torch.bfloat16)
    phi_q = torch.rand(B, H, T, m, generator=g).to(torch.bfloat16)
    la = None if kind == "sum" else torch.log(0.8 + 0.19 * torch.rand(H, generator=g, dtype=torch.float64)).float()
    eps = 1e-3
    w = torch.randn(B, H, T, m, generator=g, dtype=torch.float64)
    gk, gq = (x.to(dev).requires_grad_(True) for x in (phi_k, phi_q))
    gla = None if la is None else la.to(dev).requires_grad_(True)
    out = _MassQuery.apply(gk, gq, gla, kind == "stale", eps)
    (out.double() * w.to(dev)).sum().backward()
    ok, oq = (x.double().requires_grad_(True) for x in (phi_k, phi_q))
    ola = None if la is None else la.double().requires_grad_(True)
    want = _oracle(ok, oq, ola, kind, eps)
    (want * w).sum().backward()
    from thetascan_b200 import _lib
    assert _lib.device_status(torch.cuda.current_stream().cuda_stream) == 0
    assert rel_err(out, want) < BF16_TOL
    assert rel_err(gq.grad, oq.grad) < BF16_TOL
    assert rel_err(gk.grad, ok.grad) < BF16_TOL
    if la is not None:
        assert rel_err(gla.grad, ola.grad) < BF16_TOL


def test_mass_query_stale_first_token_is_query_over_eps(dev):
    """The stale mass of token 0 is exactly zero (its own weight 1 - alpha^0)."""
    from thetascan_b200.kernel import _MassQuery
    phi = torch.full((1, 1, 4, 16), 0.5, dtype=torch.bfloat16, device=dev)
    la = torch.tensor([math.log(0.9)], device=dev)
    out = _MassQuery.apply(phi, phi, la, True, 1e-2)
    assert torch.allclose(out[0, 0, 0].float(), torch.full((16,), 50.0, device=dev))
    # token 1: stale mass (1 - 0.9) * 0.5 = 0.05
    assert torch.allclose(out[0, 0, 1].float(), torch.full((16,), 0.5 / 0.06, device=dev), rtol=1e-2)
