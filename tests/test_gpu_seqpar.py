"""Sequence shards on the GPU: the mixer run as P contiguous T-slices, each
scanned from a zero state and corrected through the state exchange of
:mod:`thetascan_b200.seqpar`, equals the unsharded mixer.

The shards run one after another in one process (``SequentialShards``, the
single-device stand-in for the NCCL all-gather), so one autograd graph covers
all of them and the input and parameter gradients are compared too.  Both
sides are the bf16 kernel path; tolerance ``max|got - ref| / max|ref| <= 2e-2``.
"""
from __future__ import annotations

import pytest
import torch

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


def _module(kind, dev):
    from thetascan_b200.config import KernelConfig, RoPEConfig, TemporalConfig, ThetaScanConfig
    from thetascan_b200.mixer import ThetaScan
    if kind == "bspline":
        # config-4 shape in small: B-spline features (16 basis), memory 2x, and
        # a four-view bank (sum + retentions 0.9 / 0.99 / 0.999).
        cfg = ThetaScanConfig(d_model=256, n_heads=4, memory_multiplier=2, family="kernel",
                              kernel=KernelConfig(feature_map="projected_bspline", bspline_basis_count=16),
                              rope=RoPEConfig(mode="partial", fraction=0.5),
                              temporal=TemporalConfig(mode="bank", recency_branches=3,
                                                      retention_inits=(0.9, 0.99, 0.999)))
    else:
        cfg = ThetaScanConfig(d_model=256, n_heads=4, memory_multiplier=4, feature_expansion=2, family="kernel",
                              kernel=KernelConfig(feature_map="relu2_ridge"),
                              rope=RoPEConfig(mode="partial", fraction=0.5),
                              temporal=TemporalConfig(mode="bank", retention_init=0.95))
    torch.manual_seed(3)
    module = ThetaScan(cfg).to(dev)
    with torch.no_grad():
        # nonzero decode and blend so every path carries gradient
        module._core.W2[0].normal_(0.0, 0.2)
        module._core.fade_eta.normal_(0.0, 0.5)
    return module


# the last case runs the two-level tile prefix in every stage (4352-token shards)
@pytest.mark.parametrize("kind,P,T", [("bspline", 4, 512), ("relu2", 2, 384), ("relu2", 2, 8704)])
def test_sharded_mixer_matches_unsharded(dev, kind, P, T):
    from thetascan_b200.seqpar import SequentialShards
    module = _module(kind, dev)
    g = torch.Generator(device="cpu").manual_seed(5)
    x = torch.randn(2, T, 256, generator=g).to(dev).bfloat16()
    w = torch.randn(2, T, 256, generator=g).to(dev)

    xf = x.clone().requires_grad_(True)
    y_full = module(xf)
    (y_full.float() * w).sum().backward()
    ref = {n: p.grad.clone() for n, p in module.named_parameters() if p.grad is not None}
    module.zero_grad(set_to_none=True)

    xs = x.clone().requires_grad_(True)
    runner = SequentialShards(P)
    L = T // P
    y_sh = torch.cat([module(xs[:, r * L:(r + 1) * L], shard=runner.shard(r)) for r in range(P)], dim=1)
    (y_sh.float() * w).sum().backward()

    assert rel_err(y_sh, y_full) < BF16_TOL
    assert rel_err(xs.grad, xf.grad) < BF16_TOL
    for name, want in ref.items():
        got = dict(module.named_parameters())[name].grad
        assert got is not None, name
        assert rel_err(got, want) < BF16_TOL, name
