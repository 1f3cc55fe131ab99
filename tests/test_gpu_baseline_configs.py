"""GPU parity at the widths of the baseline configurations.

The other GPU tests check the kernels on small shapes; these run the mixer at
the head counts, feature widths and sequence lengths of the baseline configs:

* config 2 -- kernel family, relu2 ridge, m = 256 from 2x random feature
  expansion, partial RoPE, one fast recency branch with per-head
  alpha ~ U(0.9, 0.999), d_model 1024, 16 heads, T = 4096 (batch 1), against
  the float64 oracle mixer: output, input gradient, every parameter gradient;
* config 3 -- GN family at head_dim 128, m = 128, relu2 with the two-stage
  feature-mass read, T = 1024, against a fixture that the reference GN mixer
  produced (``tests/golden/make_golden.py``, ``gn_c3``); and config 3 as the
  baseline states it, a tanh net with damping 1e-2 and the unnormalized
  read, against the reference engine run with tanh in its nonlinearity table
  and core epsilon 1e-2 (``gn_tanh``);
* config 4 -- projected B-spline features with 16 basis functions (m = 128),
  the four-view bank (sum + 0.9 / 0.99 / 0.999), d_model 1024, 16 heads,
  T = 8192, against the float64 oracle, and the same mixer run as 4 and 8
  sequence shards (``SequentialShards``) against the unsharded run.

The module's weights are rounded to bf16-representable values first, so the
oracle and the tensor-core path read the same numbers (x is bf16 too).
Tolerance ``max|got - ref| / max|ref| <= 2e-2`` (bf16 streams, f32 state).
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
    torch.set_num_threads(os.cpu_count() or 1)
    return torch.device("cuda")


def _round_params_to_bf16(module):
    with torch.no_grad():
        for p in module.parameters():
            p.copy_(p.to(torch.bfloat16).to(p.dtype))


def _config2_module():
    from thetascan_b200.config import KernelConfig, RoPEConfig, TemporalConfig, ThetaScanConfig
    from thetascan_b200.mixer import ThetaScan
    cfg = ThetaScanConfig(d_model=1024, n_heads=16, memory_multiplier=4, feature_expansion=2, family="kernel",
                          kernel=KernelConfig(feature_map="relu2_ridge"),
                          rope=RoPEConfig(mode="partial", fraction=0.5),
                          temporal=TemporalConfig(mode="bank", retention_init=0.95))
    torch.manual_seed(0)
    module = ThetaScan(cfg)
    g = torch.Generator().manual_seed(21)
    with torch.no_grad():
        module._core.W2[0].copy_(torch.randn(module._core.W2[0].shape, generator=g) * 0.2)
        module._core.fade_eta.copy_(torch.randn(16, generator=g) * 0.5)
        alphas = 0.9 + 0.099 * torch.rand(16, generator=torch.Generator().manual_seed(0))
        module._core.fade_alpha.copy_(torch.log(alphas / (1 - alphas)))
    _round_params_to_bf16(module)
    core_cfg = {"n_heads": 16, "head_dim": 64, "feature_expansion": 2, "kernel_kind": "relu2_ridge",
                "rope": "partial", "rope_frac": 0.5, "rope_base": 10000.0, "read_fade": True,
                "read_fade_mode": "fast", "read_norm": "key_mass", "eps": 1e-6, "scan_chunk": 512}
    return module, core_cfg


def _config4_module():
    from thetascan_b200.config import KernelConfig, RoPEConfig, TemporalConfig, ThetaScanConfig
    from thetascan_b200.mixer import ThetaScan
    cfg = ThetaScanConfig(d_model=1024, n_heads=16, memory_multiplier=2, family="kernel",
                          kernel=KernelConfig(feature_map="projected_bspline", bspline_basis_count=16),
                          rope=RoPEConfig(mode="partial", fraction=0.5),
                          temporal=TemporalConfig(mode="bank", recency_branches=3,
                                                  retention_inits=(0.9, 0.99, 0.999)))
    torch.manual_seed(0)
    module = ThetaScan(cfg)
    g = torch.Generator().manual_seed(41)
    with torch.no_grad():
        module._core.W2[0].copy_(torch.randn(module._core.W2[0].shape, generator=g) * 0.2)
        module._core.fade_eta.copy_(torch.randn(module._core.fade_eta.shape, generator=g) * 0.5)
    _round_params_to_bf16(module)
    core_cfg = {"n_heads": 16, "head_dim": 64, "feature_expansion": 1, "kernel_kind": "projected_bspline",
                "bspline_basis_count": 16, "rope": "partial", "rope_frac": 0.5, "rope_base": 10000.0,
                "read_fade": True, "read_fade_mode": "fast", "read_norm": "key_mass", "eps": 1e-6,
                "scan_chunk": 512}
    return module, core_cfg


def _check_against_oracle(dev, module, core_cfg, T, seed):
    from thetascan_b200 import _lib
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(1, T, module.config.d_model, generator=g).bfloat16()
    w = torch.randn(1, T, module.config.d_model, generator=g, dtype=torch.float64)
    params = {n: t.detach().double().requires_grad_(True) for n, t in module._core.named_parameters()}
    for n, t in module._core.named_buffers():
        if n.startswith("_expand_"):
            params[n] = t.detach().double()
    gpu = module.to(dev)
    xg = x.to(dev).requires_grad_(True)
    y = gpu(xg)
    (y.double() * w.to(dev)).sum().backward()
    assert _lib.device_status(torch.cuda.current_stream().cuda_stream) == 0

    xo = x.double().requires_grad_(True)
    yo = omixer.mixer_forward(params, core_cfg, xo)
    (yo * w).sum().backward()
    assert rel_err(y, yo) < BF16_TOL
    assert rel_err(xg.grad, xo.grad) < BF16_TOL
    for name, p in gpu._core.named_parameters():
        assert rel_err(p.grad, params[name].grad) < BF16_TOL, name


def test_config2_full_width_matches_oracle(dev):
    module, core_cfg = _config2_module()
    _check_against_oracle(dev, module, core_cfg, T=4096, seed=22)


def test_config4_full_width_matches_oracle(dev):
    module, core_cfg = _config4_module()
    _check_against_oracle(dev, module, core_cfg, T=8192, seed=42)


@pytest.mark.parametrize("P", [4, 8])
def test_config4_sequence_shards_match_unsharded(dev, P):
    from thetascan_b200 import _lib
    from thetascan_b200.seqpar import SequentialShards
    module, _ = _config4_module()
    module = module.to(dev)
    T = 8192
    g = torch.Generator().manual_seed(43)
    x = torch.randn(1, T, 1024, generator=g).to(dev).bfloat16()
    w = torch.randn(1, T, 1024, generator=g).to(dev)

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
    assert _lib.device_status(torch.cuda.current_stream().cuda_stream) == 0

    assert rel_err(y_sh, y_full) < BF16_TOL
    assert rel_err(xs.grad, xf.grad) < BF16_TOL
    for name, want in ref.items():
        got = dict(module.named_parameters())[name].grad
        assert got is not None, name
        assert rel_err(got, want) < BF16_TOL, name


def test_config3_width_gn_matches_reference_fixture(dev):
    """GN at head_dim 128 and m = 128 (config 3's widths; payload 129 columns)
    on 1024 tokens, against the reference GN mixer's own output and
    gradients."""
    from thetascan_b200 import _lib
    from thetascan_b200.config import ThetaScanConfig
    from thetascan_b200.mixer import ThetaScan

    case = torch.load(os.path.join(GOLDEN, "gn_c3_cases.pt"), weights_only=False)["gn_c3_d128_T1024"]
    module = ThetaScan(ThetaScanConfig.from_dict(case["public_config"])).to(dev)
    assert module._core.head_dim == 128 and module._core.W1[0].shape[1] == 128
    module.load_state_dict({"_core." + n: t.float() for n, t in case["params"].items()
                            if not n.startswith("_expand_")})
    x = case["x"].float().to(dev).requires_grad_(True)
    y = module(x)
    (y.double() * case["out_weight"].to(dev)).sum().backward()
    assert _lib.device_status(torch.cuda.current_stream().cuda_stream) == 0
    assert rel_err(y, case["y"]) < BF16_TOL
    assert rel_err(x.grad, case["x_grad"]) < BF16_TOL
    grads = dict(module._core.named_parameters())
    for n, want in case["grads"].items():
        assert rel_err(grads[n].grad, want) < BF16_TOL, n


@pytest.mark.parametrize("name", ["gn_tanh_d128_sum", "gn_tanh_d128_bank2"])
def test_config3_tanh_gn_matches_reference_engine_fixture(dev, name):
    """The tanh GN net with damping (``GNConfig(nonlinearity="tanh",
    damping=1e-2)``, an extension of the public config) against the
    reference's own engine extended by the same table entry and epsilon."""
    from thetascan_b200 import _lib
    from thetascan_b200.config import ThetaScanConfig
    from thetascan_b200.mixer import ThetaScan

    case = torch.load(os.path.join(GOLDEN, "gn_tanh_cases.pt"), weights_only=False)[name]
    cfg = ThetaScanConfig.from_dict(case["b200_config"])
    assert cfg.gn.nonlinearity == "tanh" and cfg.gn.damping == 1e-2
    module = ThetaScan(cfg).to(dev)
    module.load_state_dict({"_core." + n: t.float() for n, t in case["params"].items()
                            if not n.startswith("_expand_")})
    x = case["x"].float().to(dev).requires_grad_(True)
    y = module(x)
    (y.double() * case["out_weight"].to(dev)).sum().backward()
    assert _lib.device_status(torch.cuda.current_stream().cuda_stream) == 0
    assert rel_err(y, case["y"]) < BF16_TOL
    assert rel_err(x.grad, case["x_grad"]) < BF16_TOL
    grads = dict(module._core.named_parameters())
    for n, want in case["grads"].items():
        assert rel_err(grads[n].grad, want) < BF16_TOL, n
