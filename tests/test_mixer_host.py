"""Host-side drop-in checks of the B200 mixer (no GPU needed).

The golden fixtures were produced by the reference module with
``torch.manual_seed(0)``; the B200 module must parse the same manifests,
expose the same state-dict names and shapes, initialise identically from the
same seed, and derive identical expansion maps and fingerprints.
"""
from __future__ import annotations

import os

import pytest
import torch

from thetascan_b200.config import ThetaScanConfig
from thetascan_b200.mixer import ThetaScan

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
CASES = ["softmax_bank_fast", "relu2_expanded_rope", "bspline_stale", "relu2_d64_ragged", "softmax_sum_feature_mass"]
# Parameters the fixture generator overwrote after construction.
OVERWRITTEN = ("W2.0", "fade_eta", "kernel_relu2_threshold")


def _fixtures():
    return torch.load(os.path.join(GOLDEN, "mixer_cases.pt"), weights_only=False)


@pytest.mark.parametrize("name", CASES)
def test_manifest_round_trip(name):
    cfg = ThetaScanConfig.from_dict(_fixtures()[name]["public_config"])
    assert ThetaScanConfig.from_dict(cfg.to_dict()) == cfg


@pytest.mark.parametrize("name", ["softmax_bank_fast", "relu2_expanded_rope", "relu2_d64_ragged", "bspline_stale",
                                  "softmax_sum_feature_mass"])
def test_state_dict_and_seeded_init_match_reference(name):
    case = _fixtures()[name]
    cfg = ThetaScanConfig.from_dict(case["public_config"])
    torch.manual_seed(0)
    module = ThetaScan(cfg)
    ours = {n[len("_core."):]: t for n, t in module.state_dict().items()}
    theirs = {n: t for n, t in case["params"].items() if not n.startswith("_expand_")}
    assert set(ours) == set(theirs)
    for n, t in ours.items():
        assert t.shape == theirs[n].shape, n
        if n not in OVERWRITTEN:
            assert torch.equal(t.to(theirs[n].dtype), theirs[n]), n
    buffers = dict(module._core.named_buffers())
    for n, t in case["params"].items():
        if n.startswith("_expand_"):
            assert torch.equal(buffers[n].to(t.dtype), t), n
    module.load_state_dict({"_core." + n: t.float() for n, t in theirs.items()})


def test_presets_and_unsupported_configs():
    kernel = ThetaScanConfig.kernel_expanded_reference_v0_1(d_model=256, n_heads=4)
    ThetaScan(kernel)  # constructs on CPU; the forward needs CUDA
    ThetaScan(ThetaScanConfig.gn_reference_v0_1(d_model=256, n_heads=4))
    ThetaScan(ThetaScanConfig.gn_expanded_reference_v0_1(d_model=256, n_heads=4))
    from thetascan_b200.config import GNConfig
    ThetaScan(ThetaScanConfig(d_model=256, n_heads=4, family="gn", gn=GNConfig(nonlinearity="swiglu"), depth=2))
    ThetaScan(ThetaScanConfig.from_dict(_fixtures()["bspline_stale"]["public_config"]))
    from thetascan_b200.config import TemporalConfig
    ThetaScan(ThetaScanConfig(d_model=256, n_heads=4, family="gn",
                              temporal=TemporalConfig(mode="bank", bank_mode="stale")))
    with pytest.raises(NotImplementedError):
        ThetaScan(ThetaScanConfig(d_model=256, n_heads=4, temporal=TemporalConfig(mode="ema")))
    with pytest.raises(ValueError):
        ThetaScanConfig(runtime=__import__("thetascan_b200.config", fromlist=["RuntimeConfig"])
                        .RuntimeConfig(backend="bogus")).validate()


def test_forward_requires_cuda():
    cfg = ThetaScanConfig.from_dict(_fixtures()["relu2_d64_ragged"]["public_config"])
    module = ThetaScan(cfg)
    with pytest.raises(RuntimeError):
        module(torch.zeros(1, 8, cfg.d_model))


GN_OVERWRITTEN = {"W2.0", "fade_eta", "Wg.0", "kq_bias"}  # set by the fixture generator


@pytest.mark.parametrize("name", ["gn_both_relu2_bank", "gn_both_threshold_expanded", "gn_w2_relu2_sum",
                                  "gn_none_silu_bank2"])
def test_gn_state_dict_and_seeded_init_match_reference(name):
    """GN modules: the same parameter names and shapes as the reference's, and
    (seed 0) the same initial values for everything the fixture generator did
    not overwrite; the reference state dict loads unchanged."""
    case = torch.load(os.path.join(GOLDEN, "gn_cases.pt"), weights_only=False)[name]
    torch.manual_seed(0)
    module = ThetaScan(ThetaScanConfig.from_dict(case["public_config"]))
    ours = {n: t for n, t in module._core.state_dict().items()}
    theirs = {n: t for n, t in case["params"].items() if not n.startswith("_expand_")}
    assert set(ours) == set(theirs)
    for n, t in ours.items():
        assert tuple(t.shape) == tuple(theirs[n].shape), n
        if n not in GN_OVERWRITTEN:
            assert torch.equal(t.to(theirs[n].dtype), theirs[n]), n
    module.load_state_dict({"_core." + n: t.float() for n, t in theirs.items()})
