"""GPU parity of the GN (Gauss--Newton fast-weight) mixer.

The module runs the GN write and features in f32 PyTorch and every sequence
read on the scan kernels (bf16 streams, f32 states).  Each case is a golden
fixture produced by the reference GN mixer itself (two-stage normalized read
with and without the learned threshold and feature expansion, the normalized
W2 read, the unnormalized silu read with a two-branch bank, and a
head_dim-64 ragged-T case): output, input gradient and every parameter
gradient.  Tolerance ``max|got - ref| / max|ref| <= 2e-2`` (bf16 streams).
"""
from __future__ import annotations

import os

import pytest
import torch

pytestmark = pytest.mark.gpu
BF16_TOL = 2e-2
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
CASES = ["gn_both_relu2_bank", "gn_both_threshold_expanded", "gn_w2_relu2_sum", "gn_none_silu_bank2",
         "gn_d64_ragged", "gn_d64_stale"]


def rel_err(got, want):
    got = got.detach().to("cpu", torch.float64)
    want = want.detach().to("cpu", torch.float64)
    return float((got - want).abs().max() / want.abs().max().clamp_min(1e-30))


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda")


@pytest.mark.parametrize("name", CASES)
def test_gn_mixer_matches_reference_fixture(dev, name):
    from thetascan_b200 import _lib
    from thetascan_b200.config import ThetaScanConfig
    from thetascan_b200.mixer import ThetaScan

    case = torch.load(os.path.join(GOLDEN, "gn_cases.pt"), weights_only=False)[name]
    module = ThetaScan(ThetaScanConfig.from_dict(case["public_config"])).to(dev)
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


# The write of two Jacobian steps matches float64 autograd at 1e-5 on its own
# (tests/test_gpu_gn_rows.py, two-step write); the reads scan twice the
# streams (two g payloads, two lambda streams with their own keys), all bf16,
# and the thresholded case's W1 gradient lands at 2.1% of its largest entry.
JAC2_LOOSE = {("gn_jac2_threshold_sum", "W1.0"): 3e-2}


@pytest.mark.parametrize("name", ["gn_jac2_relu2_bank", "gn_jac2_threshold_sum"])
def test_gn_two_jacobian_steps_match_reference_fixture(dev, name):
    """Two Jacobian steps of the write (``GNConfig(jacobian_steps=2)``, the
    reference's ``write_iters == 2``, engine.py:323-339) with unnormalized
    reads, against fixtures of the reference GN mixer: output, input
    gradient, every parameter gradient."""
    from thetascan_b200 import _lib
    from thetascan_b200.config import ThetaScanConfig
    from thetascan_b200.mixer import ThetaScan

    case = torch.load(os.path.join(GOLDEN, "gn_jac2_cases.pt"), weights_only=False)[name]
    module = ThetaScan(ThetaScanConfig.from_dict(case["public_config"])).to(dev)
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
        assert rel_err(grads[n].grad, want) < JAC2_LOOSE.get((name, n), BF16_TOL), n


DEEP_CASES = ["gn_swiglu_sum", "gn_swiglu_jac2_bank", "gn_depth2_both_bank", "gn_depth2_swiglu_stale",
              "gn_depth3_threshold_w2_expanded", "gn_depth2_silu_jac2_bank2"]


# gn_deep runs float32 end to end (plain f32 projections, f32 scan kernels);
# the fixtures' retention gradients move by 1-2% under a 2^-11 relative
# perturbation of q and k alone, so TF32 or bf16 operands could not be told
# apart from a wrong result here.
DEEP_TOL = 2e-3


@pytest.mark.parametrize("name", DEEP_CASES)
def test_gn_deep_and_swiglu_match_reference_fixture(dev, name):
    """GN nets of depth 2 and 3 and the swiglu activation (``gn_deep``: the
    per-token maps in f32, every read on the float32 scan kernels), with one
    and two Jacobian steps, each read normalisation, fast and stale banks,
    against fixtures of the reference GN mixer: output, input gradient, every
    parameter gradient."""
    from thetascan_b200 import _lib
    from thetascan_b200.config import ThetaScanConfig
    from thetascan_b200.mixer import ThetaScan

    case = torch.load(os.path.join(GOLDEN, "gn_deep_cases.pt"), weights_only=False)[name]
    module = ThetaScan(ThetaScanConfig.from_dict(case["public_config"])).to(dev)
    module.load_state_dict({"_core." + n: t.float() for n, t in case["params"].items()
                            if not n.startswith("_expand_")})
    before = _lib.load().ts_b200_launch_count()
    x = case["x"].float().to(dev).requires_grad_(True)
    y = module(x)
    (y.double() * case["out_weight"].to(dev)).sum().backward()
    torch.cuda.synchronize()
    assert _lib.load().ts_b200_launch_count() > before   # the reads ran on the library kernels
    assert _lib.device_status(torch.cuda.current_stream().cuda_stream) == 0
    errs = {"y": rel_err(y, case["y"]), "x": rel_err(x.grad, case["x_grad"])}
    grads = dict(module._core.named_parameters())
    for n, want in case["grads"].items():
        errs[n] = rel_err(grads[n].grad, want)
    worst = max(errs, key=errs.get)
    assert errs[worst] < DEEP_TOL, (worst, errs)
