"""``thetascan_b200.integration.install`` registers backend "b200" in an
installed reference package (CPU checks of the routing; skipped where the
reference package is not importable, see ``tests/_refpkg.py``)."""
from __future__ import annotations

import os
import sys

import pytest
import torch

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from _refpkg import import_reference  # noqa: E402


@pytest.fixture(scope="module")
def thetascan():
    ts = import_reference()
    from thetascan_b200 import integration
    integration.install()
    return ts


def test_backend_name_validates(thetascan):
    from thetascan import KernelConfig, RuntimeConfig, ThetaScanConfig
    cfg = ThetaScanConfig(family="kernel", kernel=KernelConfig(feature_map="relu2_ridge"),
                          runtime=RuntimeConfig(backend="b200", scan_chunk=128))
    cfg.validate()
    core = cfg._to_core_config()
    assert core.backend == "b200"
    with pytest.raises(ValueError):
        ThetaScanConfig(runtime=RuntimeConfig(backend="nope")).validate()


def test_cpu_input_raises_like_the_reference_cuda_backends(thetascan):
    from thetascan import KernelConfig, RuntimeConfig, ThetaScan, ThetaScanConfig
    cfg = ThetaScanConfig(d_model=64, n_heads=2, family="kernel",
                          kernel=KernelConfig(feature_map="relu2_ridge"),
                          runtime=RuntimeConfig(backend="b200"))
    module = ThetaScan(cfg)
    with pytest.raises(RuntimeError):
        module(torch.zeros(1, 8, 64))


def test_scan_plugin_point_routes_b200(thetascan):
    from thetascan._core.ops import interface
    fn = interface._fn("b200", 64)
    q = torch.zeros(1, 2, 8, 4)
    with pytest.raises(RuntimeError):
        fn(q, q, q)
    # Other backends are untouched.
    assert interface._fn("chunk", 64).func.__module__.endswith("scan_chunk")


def test_fused_view_shares_parameters(thetascan):
    from thetascan import KernelConfig, RoPEConfig, RuntimeConfig, TemporalConfig, ThetaScan, ThetaScanConfig
    from thetascan_b200 import integration
    cfg = ThetaScanConfig(d_model=128, n_heads=2, memory_multiplier=4, feature_expansion=2, family="kernel",
                          kernel=KernelConfig(feature_map="relu2_ridge"), rope=RoPEConfig(mode="partial"),
                          temporal=TemporalConfig(mode="bank"), runtime=RuntimeConfig(backend="b200"))
    module = ThetaScan(cfg)
    state = torch.random.get_rng_state()
    fused = integration._fused_core(module._core)
    assert torch.equal(state, torch.random.get_rng_state())
    assert fused is not None
    assert fused.W1[0] is module._core.W1[0]
    assert fused.proj_qkv.weight is module._core.proj_qkv.weight
    assert fused._expand_w1_0 is module._core._expand_w1_0
