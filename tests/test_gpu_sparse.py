"""GPU parity of the relative sparsity of the softmax partition
(kernel_features.py:43-113 of the reference: relative_soft, relative_st,
relative_st_blend) against mixers of the reference itself
(``tests/golden/sparse_cases.pt``, head_dim 64, m = 128, fast bank):

* bf16 input: the fused feature kernels (``TS_SPARSITY_*`` of
  ``ts_feature_args``) on the tensor-core path, ``max|got - ref| / max|ref|
  <= 2e-2`` on the output, the input gradient and every parameter gradient
  (the cutoff and the blend included);
* float32 input: the float32 path (per-token maps in float32, the float32
  scan kernels), bound 1e-4 against the float64 fixture evaluated at float64
  inputs.
"""
from __future__ import annotations

import os

import pytest
import torch

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
MODES = ["relative_soft", "relative_st", "relative_st_blend"]


def rel_err(got, want):
    got = got.detach().to("cpu", torch.float64)
    want = want.detach().to("cpu", torch.float64)
    return float((got - want).abs().max() / want.abs().max().clamp_min(1e-30))


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda")


def _run(dev, name, dtype):
    from thetascan_b200 import _lib
    from thetascan_b200.config import ThetaScanConfig
    from thetascan_b200.mixer import ThetaScan
    case = torch.load(os.path.join(GOLDEN, "sparse_cases.pt"), weights_only=False)["mixers"][name]
    module = ThetaScan(ThetaScanConfig.from_dict(case["public_config"])).to(dev)
    module.load_state_dict({"_core." + n: t.float() for n, t in case["params"].items()
                            if not n.startswith("_expand_")})
    x = case["x"].to(dev, dtype).requires_grad_(True)
    y = module(x)
    (y.double() * case["out_weight"].to(dev)).sum().backward()
    assert _lib.device_status(torch.cuda.current_stream().cuda_stream) == 0
    return case, module, x, y


@pytest.mark.parametrize("mode", MODES)
def test_sparse_mixer_bf16_matches_reference(dev, mode):
    case, module, x, y = _run(dev, f"softmax_{mode}", torch.bfloat16)
    assert rel_err(y, case["y"]) < 2e-2
    assert rel_err(x.grad, case["x_grad"]) < 2e-2
    grads = dict(module._core.named_parameters())
    for n, want in case["grads"].items():
        assert rel_err(grads[n].grad, want) < 2e-2, n


@pytest.mark.parametrize("mode", MODES)
def test_sparse_mixer_f32_matches_reference(dev, mode):
    case, module, x, y = _run(dev, f"softmax_{mode}", torch.float32)
    assert rel_err(y, case["y"]) < 1e-4
    assert rel_err(x.grad, case["x_grad"]) < 1e-4
    grads = dict(module._core.named_parameters())
    for n, want in case["grads"].items():
        assert rel_err(grads[n].grad, want) < 1e-4, n
