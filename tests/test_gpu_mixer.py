"""GPU parity of the whole B200 mixer (projections, RoPE, hot path, gate).

1. Against the committed golden fixture produced by the reference module
   itself (``relu2_d64_ragged``: relu2 ridge, partial RoPE, fast bank,
   ragged T=160): output, input gradient and every parameter gradient.
2. Against the float64 oracle mixer on a config-2-shaped module (relu2 ridge
   with 2x random feature expansion, m=256, partial RoPE, fast bank).
Tolerance: ``max|got - ref| / max|ref| <= 2e-2`` (bf16 streams).
"""
from __future__ import annotations

import os

import pytest
import torch

from oracle import mixer as omixer

pytestmark = pytest.mark.gpu
BF16_TOL = 2e-2
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def rel_err(got, want):
    got = got.detach().to("cpu", torch.float64)
    want = want.detach().to("cpu", torch.float64)
    return float((got - want).abs().max() / want.abs().max().clamp_min(1e-30))


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda")


def test_mixer_matches_reference_golden_fixture(dev):
    from thetascan_b200.config import ThetaScanConfig
    from thetascan_b200.mixer import ThetaScan

    case = torch.load(os.path.join(GOLDEN, "mixer_cases.pt"), weights_only=False)["relu2_d64_ragged"]
    module = ThetaScan(ThetaScanConfig.from_dict(case["public_config"])).to(dev)
    state = {"_core." + n: t.float() for n, t in case["params"].items() if not n.startswith("_expand_")}
    module.load_state_dict(state)
    x = case["x"].float().to(dev).requires_grad_(True)
    y = module(x)
    assert rel_err(y, case["y"]) < BF16_TOL
    (y.double() * case["out_weight"].to(dev)).sum().backward()
    assert rel_err(x.grad, case["x_grad"]) < BF16_TOL
    grads = dict(module._core.named_parameters())
    for name, want in case["grads"].items():
        assert rel_err(grads[name].grad, want) < BF16_TOL, name


def test_config2_shaped_mixer_matches_oracle(dev):
    from thetascan_b200.config import KernelConfig, RoPEConfig, TemporalConfig, ThetaScanConfig
    from thetascan_b200.mixer import ThetaScan

    cfg = ThetaScanConfig(d_model=256, n_heads=4, memory_multiplier=4, feature_expansion=2, family="kernel",
                          kernel=KernelConfig(feature_map="relu2_ridge"),
                          rope=RoPEConfig(mode="partial", fraction=0.5),
                          temporal=TemporalConfig(mode="bank", retention_init=0.95))
    torch.manual_seed(0)
    module = ThetaScan(cfg)
    with torch.no_grad():
        g = torch.Generator().manual_seed(3)
        module._core.W2[0].copy_(torch.randn(module._core.W2[0].shape, generator=g) * 0.2)
        module._core.fade_eta.copy_(torch.randn(4, generator=g) * 0.5)
        alphas = 0.9 + 0.099 * torch.rand(4, generator=g)
        module._core.fade_alpha.copy_(torch.log(alphas / (1 - alphas)))
    module = module.to(dev)
    B, T = 2, 600
    x = torch.randn(B, T, 256, generator=torch.Generator().manual_seed(4))
    xg = x.to(dev).requires_grad_(True)
    y = module(xg)
    w = torch.randn(B, T, 256, generator=torch.Generator().manual_seed(5), dtype=torch.float64)
    (y.double() * w.to(dev)).sum().backward()

    core_cfg = {"n_heads": 4, "head_dim": 64, "feature_expansion": 2, "kernel_kind": "relu2_ridge",
                "rope": "partial", "rope_frac": 0.5, "rope_base": 10000.0, "read_fade": True,
                "read_fade_mode": "fast", "read_norm": "key_mass", "eps": 1e-6, "scan_chunk": 128}
    params = {n: t.detach().cpu().double().requires_grad_(True) for n, t in module._core.named_parameters()}
    for n, t in module._core.named_buffers():
        if n.startswith("_expand_"):
            params[n] = t.detach().cpu().double()
    xo = x.double().requires_grad_(True)
    yo = omixer.mixer_forward(params, core_cfg, xo)
    (yo * w).sum().backward()
    assert rel_err(y, yo) < BF16_TOL
    assert rel_err(xg.grad, xo.grad) < BF16_TOL
    for name, p in module._core.named_parameters():
        assert rel_err(p.grad, params[name].grad) < BF16_TOL, name
