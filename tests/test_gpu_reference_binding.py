"""The reference package itself with ``backend="b200"``, on the GPU.

``thetascan_b200.integration.install()`` registers the backend inside the
reference ``thetascan`` package (found as ``tests/_refpkg.py`` says).  Each
test builds the reference's own public ``ThetaScan`` twice from one config --
``backend="b200"`` on the GPU, and the reference's default ``chunk`` backend
in float64 on the CPU with the same weights -- and compares output, input
gradient and every parameter gradient:

* a kernel-family config (relu2 ridge, m = 256 from 2x expansion, partial
  RoPE, fast bank): the fused b200 mixer replaces the reference forward;
  bf16 input, tolerance 2e-2;
* a GN-family config (two-stage feature-mass read, fast bank): the reference
  forward runs unchanged and its scans go through the scan-level plugin
  point (``interface.scan_views`` / ``_fn``) to the float32 scan kernels;
  float32 input, tolerance 1e-4.
"""
from __future__ import annotations

import copy
import os
import sys

import pytest
import torch

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from _refpkg import import_reference  # noqa: E402

pytestmark = pytest.mark.gpu


def rel_err(got, want):
    got = got.detach().to("cpu", torch.float64)
    want = want.detach().to("cpu", torch.float64)
    return float((got - want).abs().max() / want.abs().max().clamp_min(1e-30))


@pytest.fixture(scope="module")
def ref():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    ts = import_reference()
    from thetascan_b200 import integration
    integration.install()
    return ts


def _pair(ts, cfg_b200, seed):
    from thetascan import RuntimeConfig
    torch.manual_seed(seed)
    module = ts.ThetaScan(cfg_b200)
    core = module._core
    g = torch.Generator().manual_seed(seed + 1)
    with torch.no_grad():
        for p in core.W2:
            p.copy_(torch.randn(p.shape, generator=g) * 0.2)
        if getattr(core, "fade_eta", None) is not None:
            core.fade_eta.copy_(torch.randn(core.fade_eta.shape, generator=g) * 0.5)
        for p in module.parameters():
            p.copy_(p.to(torch.bfloat16).to(p.dtype))   # bf16-representable weights
    cfg_chunk = copy.deepcopy(cfg_b200)
    cfg_chunk.runtime = RuntimeConfig(backend="chunk", scan_chunk=cfg_b200.runtime.scan_chunk)
    reference = ts.ThetaScan(cfg_chunk)
    reference.load_state_dict(module.state_dict())
    return module, reference.double()


def _compare(module, reference, x, dtype, dev, tol):
    w = torch.randn(x.shape, generator=torch.Generator().manual_seed(99), dtype=torch.float64)
    gpu = module.to(dev)
    xg = x.to(dev, dtype).requires_grad_(True)
    y = gpu(xg)
    assert y.is_cuda
    (y.double() * w.to(dev)).sum().backward()
    xr = x.to(dtype).double().requires_grad_(True)
    yr = reference(xr)
    (yr * w).sum().backward()
    assert rel_err(y, yr) < tol
    assert rel_err(xg.grad, xr.grad) < tol
    want = dict(reference.named_parameters())
    for name, p in gpu.named_parameters():
        assert p.grad is not None, name
        assert rel_err(p.grad, want[name].grad) < tol, name


def test_reference_kernel_mixer_on_b200_matches_reference_chunk(ref):
    from thetascan import KernelConfig, RoPEConfig, RuntimeConfig, TemporalConfig, ThetaScanConfig
    cfg = ThetaScanConfig(d_model=256, n_heads=4, memory_multiplier=4, feature_expansion=2, family="kernel",
                          kernel=KernelConfig(feature_map="relu2_ridge"),
                          rope=RoPEConfig(mode="partial", fraction=0.5),
                          temporal=TemporalConfig(mode="bank", retention_init=0.95),
                          runtime=RuntimeConfig(backend="b200", scan_chunk=128))
    module, reference = _pair(ref, cfg, seed=5)
    from thetascan_b200 import integration
    assert integration._fused_core(module._core) is not None   # the fused mixer runs
    x = torch.randn(2, 600, 256, generator=torch.Generator().manual_seed(6))
    _compare(module, reference, x, torch.bfloat16, torch.device("cuda"), 2e-2)


def test_reference_gn_mixer_scans_on_b200_match_reference_chunk(ref):
    from thetascan import GNConfig, RoPEConfig, RuntimeConfig, TemporalConfig, ThetaScanConfig
    cfg = ThetaScanConfig(d_model=128, n_heads=2, memory_multiplier=2, family="gn",
                          gn=GNConfig(nonlinearity="relu2", read_normalization="both_feature_mass"),
                          rope=RoPEConfig(mode="partial", fraction=0.5),
                          temporal=TemporalConfig(mode="bank", retention_init=0.9),
                          runtime=RuntimeConfig(backend="b200", scan_chunk=64))
    module, reference = _pair(ref, cfg, seed=7)
    from thetascan_b200 import integration
    assert integration._fused_core(module._core) is None   # reference forward, b200 scans
    x = torch.randn(2, 300, 128, generator=torch.Generator().manual_seed(8))
    _compare(module, reference, x, torch.float32, torch.device("cuda"), 1e-4)


def test_reference_scan_plugin_point_takes_retention_streams(ref):
    """The reference's scan plugin point (``interface._fn``) with a per-token
    ``[B,H,T,1]`` log-retention stream: ``backend="b200"`` on float32 CUDA
    tensors against the reference's own chunk scan in float64."""
    from thetascan._core.ops import interface, scan_chunk
    g = torch.Generator().manual_seed(21)
    B, H, T, Dk, Dv = 2, 3, 700, 48, 40
    q, k = (torch.randn(B, H, T, Dk, generator=g).abs() / Dk ** 0.5 for _ in range(2))
    v = torch.randn(B, H, T, Dv, generator=g)
    decay = torch.nn.functional.logsigmoid(torch.randn(B, H, T, 1, generator=g) + 4.0)
    w = torch.randn(B, H, T, Dv, generator=g, dtype=torch.float64)
    leaves = [x.cuda().requires_grad_(True) for x in (q, k, v, decay)]
    y = interface._fn("b200", 128)(*leaves)
    (y.double() * w.cuda()).sum().backward()
    rleaves = [x.double().requires_grad_(True) for x in (q, k, v, decay)]
    yr = scan_chunk.linattn(*rleaves, chunk=128)
    (yr * w).sum().backward()
    assert y.dtype == torch.float32
    assert rel_err(y, yr) < 1e-5
    for a, b in zip(leaves, rleaves):
        assert rel_err(a.grad, b.grad) < 1e-5


def test_reference_ema_mixer_scans_on_b200_match_reference_chunk(ref):
    """The reference's data-dependent EMA mode (``TemporalConfig(mode="ema")``:
    a decay gate makes per-token ``[B,H,T,1]`` log-retention streams for the
    numerator scan and the key mass, interface.py:198-230) with
    ``backend="b200"``: the reference forward runs unchanged and its stream
    scans go through the plugin point to the float32 stream kernels."""
    from thetascan import KernelConfig, RoPEConfig, RuntimeConfig, TemporalConfig, ThetaScanConfig
    cfg = ThetaScanConfig(d_model=128, n_heads=2, memory_multiplier=2, family="kernel",
                          kernel=KernelConfig(feature_map="relu2_ridge"),
                          rope=RoPEConfig(mode="partial", fraction=0.5),
                          temporal=TemporalConfig(mode="ema"),
                          runtime=RuntimeConfig(backend="b200", scan_chunk=64))
    module, reference = _pair(ref, cfg, seed=9)
    from thetascan_b200 import integration
    assert integration._fused_core(module._core) is None   # reference forward, b200 stream scans
    x = torch.randn(2, 300, 128, generator=torch.Generator().manual_seed(10))
    _compare(module, reference, x, torch.float32, torch.device("cuda"), 1e-4)
