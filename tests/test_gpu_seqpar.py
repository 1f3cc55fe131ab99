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


def _views_module(kind, dev):
    """Configurations whose shards take the float32 path: a stale bank, the
    per-feature mass read, and the GN family."""
    from thetascan_b200.config import GNConfig, KernelConfig, RoPEConfig, TemporalConfig, ThetaScanConfig
    from thetascan_b200.mixer import ThetaScan
    rope = RoPEConfig(mode="partial", fraction=0.5)
    if kind == "stale":
        cfg = ThetaScanConfig(d_model=256, n_heads=4, memory_multiplier=2, family="kernel",
                              kernel=KernelConfig(feature_map="projected_bspline", bspline_basis_count=16), rope=rope,
                              temporal=TemporalConfig(mode="bank", bank_mode="stale", recency_branches=2,
                                                      retention_inits=(0.9, 0.99)))
    elif kind == "feature_mass":
        cfg = ThetaScanConfig(d_model=256, n_heads=4, memory_multiplier=2, family="kernel",
                              kernel=KernelConfig(feature_map="relu2_ridge", read_normalization="feature_mass"),
                              rope=rope, temporal=TemporalConfig(mode="bank", retention_init=0.95))
    else:
        gn = GNConfig(nonlinearity="relu2", read_normalization="both_feature_mass") if kind == "gn_both" else \
            GNConfig(nonlinearity="swiglu", jacobian_steps=2)
        # A stale view read with a normalisation divides the difference of
        # two reads by eps at the first token, where both are ~0 (0/0 in the
        # reference's formulation too, FadeStale = sum - fast): its gradient
        # there is rounding noise / eps and differs between any two
        # evaluations.  The normalised GN read shards with a fast bank; the
        # stale bank is covered by the unnormalised swiglu net.
        bank = "fast" if kind == "gn_both" else "stale"
        cfg = ThetaScanConfig(d_model=256, n_heads=4, memory_multiplier=2, family="gn", gn=gn, rope=rope,
                              depth=2 if kind == "gn_swiglu" else 1,
                              temporal=TemporalConfig(mode="bank", bank_mode=bank, retention_init=0.9))
    torch.manual_seed(3)
    module = ThetaScan(cfg).to(dev)
    with torch.no_grad():
        for p in module._core.W2:
            p.normal_(0.0, 0.2)
        module._core.fade_eta.normal_(0.0, 0.5)
    return module


# Both sides run the same float32 arithmetic; the sharded one adds the
# exchange's GEMMs and sums in another order, and a stale view is the
# difference of two reads, which amplifies that: the stale B-spline bank's
# input gradient lands at 1.5e-4.  The bound is float32 accumulation, not bf16.
F32_SHARD_TOL = 1e-3


@pytest.mark.parametrize("kind,P", [("stale", 2), ("feature_mass", 4), ("gn_both", 2), ("gn_swiglu", 2)])
def test_sharded_views_match_unsharded(dev, kind, P):
    """Stale banks, the per-feature mass read and the GN family (two-stage
    read with a fast bank; swiglu with two Jacobian steps at depth 2 and a
    stale bank) as sequence shards: the float32 path of every shard, each scan entering with the
    earlier shards' state (``seqpar.sharded_reads``), against the same
    module on the whole sequence -- output, input gradient, every parameter
    gradient (the whole sequence run as a single shard takes the same
    float32 path)."""
    from thetascan_b200.seqpar import SequentialShards
    module = _views_module(kind, dev)
    T = 256
    g = torch.Generator(device="cpu").manual_seed(7)
    x = torch.randn(2, T, 256, generator=g).to(dev)
    w = torch.randn(2, T, 256, generator=g).to(dev)

    # the whole sequence as one shard: the same float32 path, no exchange
    xf = x.clone().requires_grad_(True)
    y_full = module(xf, shard=SequentialShards(1).shard(0))
    (y_full * w).sum().backward()
    ref = {n: p.grad.clone() for n, p in module.named_parameters() if p.grad is not None}
    module.zero_grad(set_to_none=True)

    xs = x.clone().requires_grad_(True)
    runner = SequentialShards(P)
    L = T // P
    y_sh = torch.cat([module(xs[:, r * L:(r + 1) * L], shard=runner.shard(r)) for r in range(P)], dim=1)
    (y_sh * w).sum().backward()

    assert rel_err(y_sh, y_full) < F32_SHARD_TOL
    assert rel_err(xs.grad, xf.grad) < F32_SHARD_TOL
    for name, want in ref.items():
        got = dict(module.named_parameters())[name].grad
        assert got is not None, name
        assert rel_err(got, want) < F32_SHARD_TOL, name
