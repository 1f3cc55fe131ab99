"""GPU parity of the fused kernel-family hot path (features -> scan -> read).

Compared with ``oracle.mixer.kernel_core`` (float64 CPU, pinned to the
reference) on outputs and on the gradients of every input and parameter.
Tolerance: ``max|got - ref| / max|ref| <= 2e-2`` (bf16 streams, f32 state).
"""
from __future__ import annotations

import math

import pytest
import torch
import torch.nn.functional as F

from oracle import mixer as omixer

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


CASES = {
    # name: (kind, P, basis, mode, J, B, H, T, d)
    "relu2_m256_fast": ("relu2_ridge", 256, 1, "fast", 1, 2, 2, 300, 64),
    "relu2_m128_sum": ("relu2_ridge", 128, 1, "sum", 0, 1, 2, 200, 64),
    "softmax_m64_fast2": ("softmax_partition", 64, 1, "fast", 2, 2, 2, 257, 64),
    "bspline_p8x16_fast3": ("projected_bspline", 8, 16, "fast", 3, 1, 2, 384, 64),
}


def _case_tensors(name):
    kind, P, basis, mode, J, B, H, T, d = CASES[name]
    g = torch.Generator().manual_seed(sum(map(ord, name)))
    q = F.normalize(torch.randn(B, H, T, d, generator=g), dim=-1).to(torch.bfloat16)
    k = F.normalize(torch.randn(B, H, T, d, generator=g), dim=-1).to(torch.bfloat16)
    v = torch.randn(B, H, T, d, generator=g).to(torch.bfloat16)
    m = P * basis
    W1 = torch.randn(H, P, d, generator=g) / math.sqrt(d)
    W2 = torch.randn(H, d, m, generator=g) * 0.2
    ctl = {}
    if kind == "relu2_ridge":
        ctl["threshold"] = torch.randn(H, generator=g) * 0.1
    elif kind == "softmax_partition":
        ctl["gain"] = 4.0 + 8.0 * torch.rand(H, generator=g)
    else:
        ctl["spline_scale"] = 0.5 + torch.rand(H, generator=g)
    log_alphas = etas = None
    if J:
        alphas = torch.empty(J, H)
        for j in range(J):
            alphas[j] = 0.9 + 0.099 * torch.rand(H, generator=g)
        log_alphas = alphas.log()
        etas = torch.randn(J, H, generator=g) * 0.5
    w_out = torch.randn(B, T, H, d, generator=g, dtype=torch.float64)
    return kind, basis, mode, q, k, v, W1, W2, ctl, log_alphas, etas, w_out


@pytest.mark.parametrize("name", list(CASES))
def test_kernel_core_matches_oracle_forward_and_backward(dev, name):
    from thetascan_b200 import _lib
    from thetascan_b200.kernel import KernelSpec, kernel_core

    kind, basis, mode, q, k, v, W1, W2, ctl, las, etas, w_out = _case_tensors(name)
    spec = KernelSpec(kind=kind, mode=mode, basis=basis)

    def leaf(x, dtype=None):
        return None if x is None else x.to(dev, dtype or x.dtype).clone().requires_grad_(True)

    gq, gk, gv, gW1, gW2 = (leaf(x) for x in (q, k, v, W1, W2))
    gctl = {key: leaf(val) for key, val in ctl.items()}
    gla, geta = leaf(las), leaf(etas)
    y = kernel_core(gq, gk, gv, gW1, gW2, spec, threshold=gctl.get("threshold"), gain=gctl.get("gain"),
                    spline_scale=gctl.get("spline_scale"), log_alphas=gla, etas=geta)
    (y.double() * w_out.to(dev)).sum().backward()
    assert _lib.device_status(torch.cuda.current_stream().cuda_stream) == 0

    oq, ok_, ov = (x.double().requires_grad_(True) for x in (q, k, v))
    oW1, oW2 = W1.double().requires_grad_(True), W2.double().requires_grad_(True)
    octl = {key: val.double().requires_grad_(True) for key, val in ctl.items()}
    ola = None if las is None else las.double().requires_grad_(True)
    oeta = None if etas is None else etas.double().requires_grad_(True)
    spec_dict = {"kind": kind}
    if kind == "relu2_ridge":
        spec_dict["relu2_threshold"] = octl["threshold"]
    elif kind == "softmax_partition":
        spec_dict["gain"] = octl["gain"]
    else:
        spec_dict.update(n_basis=basis, scale=octl["spline_scale"])
    want = omixer.kernel_core(oq, ok_, ov, oW1, oW2, spec_dict, log_alphas=ola, etas=oeta, mode=mode,
                              chunk=64)
    (want.transpose(1, 2) * w_out).sum().backward()

    assert rel_err(y, want.transpose(1, 2)) < BF16_TOL
    pairs = [("q", gq, oq), ("k", gk, ok_), ("v", gv, ov), ("W1", gW1, oW1), ("W2", gW2, oW2)]
    pairs += [(key, gctl[key], octl[key]) for key in ctl]
    if las is not None:
        pairs += [("log_alpha", gla, ola), ("eta", geta, oeta)]
    for label, got, ref in pairs:
        assert rel_err(got.grad, ref.grad) < BF16_TOL, label


def test_stale_bank_is_rejected_explicitly(dev):
    """The stale view is not implemented on the GPU path yet; it must raise,
    never silently compute a low-precision difference of scans."""
    from thetascan_b200.kernel import KernelSpec, kernel_core
    q = torch.zeros(1, 2, 8, 64, dtype=torch.bfloat16, device=dev)
    W1 = torch.zeros(2, 64, 64, device=dev)
    W2 = torch.zeros(2, 64, 64, device=dev)
    with pytest.raises(NotImplementedError):
        kernel_core(q, q, q, W1, W2, KernelSpec(kind="softmax_partition", mode="stale"),
                    log_alphas=torch.zeros(1, 2, device=dev), etas=torch.zeros(1, 2, device=dev))
