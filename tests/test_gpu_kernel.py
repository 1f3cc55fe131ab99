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
    # per-feature controls: score bias with a threshold, per-feature sharpness with a bias
    "relu2_bias_threshold": ("relu2_ridge", 128, 1, "fast", 1, 1, 2, 200, 64),
    "softmax_feature_gain_bias": ("softmax_partition", 64, 1, "sum", 0, 1, 2, 150, 64),
    # stale banks: slots 1..J are stale scans (weights 1 - alpha^(t-i))
    "relu2_m256_stale": ("relu2_ridge", 256, 1, "stale", 1, 2, 2, 300, 64),
    "softmax_m64_stale2": ("softmax_partition", 64, 1, "stale", 2, 1, 2, 257, 64),
    "bspline_p8x16_stale3": ("projected_bspline", 8, 16, "stale", 3, 1, 2, 384, 64),
    # feature-mass and unnormalized reads (engine.py:402-416, 443-456)
    "softmax_m64_fm_sum": ("softmax_partition", 64, 1, "sum", 0, 1, 2, 200, 64),
    "relu2_m128_fm_fast": ("relu2_ridge", 128, 1, "fast", 1, 1, 2, 300, 64),
    "bspline_p8x16_fm_stale2": ("projected_bspline", 8, 16, "stale", 2, 1, 2, 257, 64),
    "relu2_m128_none_fast2": ("relu2_ridge", 128, 1, "fast", 2, 1, 2, 300, 64),
    "softmax_m64_none_stale": ("softmax_partition", 64, 1, "stale", 1, 1, 2, 200, 64),
}
READ = {"softmax_m64_fm_sum": "feature_mass", "relu2_m128_fm_fast": "feature_mass",
        "bspline_p8x16_fm_stale2": "feature_mass",
        "relu2_m128_none_fast2": "none", "softmax_m64_none_stale": "none"}
EPS: dict[str, float] = {}
WITH_BIAS = {"relu2_bias_threshold", "softmax_feature_gain_bias"}
# The stale view's log-retention gradient of this case is small by
# cancellation (-1.8 against terms of ~30-50 in the fast cases): rounding the
# read gradient handed to the scan to bf16 -- and nothing else -- moves the
# float64 value by 2.3% (tests/test_conditioning.py), so no bf16 hand-over can
# meet 2e-2 on it.  Its outputs and every other gradient are checked; the
# stale log-retention gradient is checked on the other stale cases.
ILL_CONDITIONED_RETENTION = {"relu2_m256_stale"}
# Feature mass with a stale view: where a feature's stale mass is below eps
# the view's query is ~phi_q / eps (~1e5 here), and the scan and mass parts of
# the log-retention gradient are large terms that must cancel.  A bf16
# quotient leaves 2-10% of the result, so that view keeps its quotient in f32
# and scans it on float32 streams; its log-retention gradient is checked at
# 2e-2 with the rest.
OPEN_PRECISION_RETENTION: set[str] = set()


def _case_tensors(name):
    kind, P, basis, mode, J, B, H, T, d = CASES[name]
    g = torch.Generator().manual_seed(sum(map(ord, name)))
    q = F.normalize(torch.randn(B, H, T, d, generator=g), dim=-1).to(torch.bfloat16)
    k = F.normalize(torch.randn(B, H, T, d, generator=g), dim=-1).to(torch.bfloat16)
    v = torch.randn(B, H, T, d, generator=g).to(torch.bfloat16)
    m = P * basis
    # Weights are bf16-representable: the kernels take bf16 projection
    # operands, so the oracle sees the same values (rounding W1 to bf16 moves
    # the logits of a sharp softmax by up to gain * |a| * 2^-9).
    W1 = (torch.randn(H, P, d, generator=g) / math.sqrt(d)).bfloat16().float()
    W2 = (torch.randn(H, d, m, generator=g) * 0.2).bfloat16().float()
    ctl = {}
    if kind == "relu2_ridge":
        ctl["threshold"] = torch.randn(H, generator=g) * 0.1
    elif kind == "softmax_partition":
        shape = (H, m) if name in WITH_BIAS else (H,)
        ctl["gain"] = 4.0 + 8.0 * torch.rand(*shape, generator=g)
    else:
        ctl["spline_scale"] = 0.5 + torch.rand(H, generator=g)
    if name in WITH_BIAS:
        ctl["score_bias"] = torch.randn(H, m, generator=g) * 0.2
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
    spec = KernelSpec(kind=kind, mode=mode, basis=basis, read=READ.get(name, "key_mass"), eps=EPS.get(name, 1e-6))

    def leaf(x, dtype=None):
        return None if x is None else x.to(dev, dtype or x.dtype).clone().requires_grad_(True)

    gq, gk, gv, gW1, gW2 = (leaf(x) for x in (q, k, v, W1, W2))
    gctl = {key: leaf(val) for key, val in ctl.items()}
    gla, geta = leaf(las), leaf(etas)
    y = kernel_core(gq, gk, gv, gW1, gW2, spec, threshold=gctl.get("threshold"), gain=gctl.get("gain"),
                    spline_scale=gctl.get("spline_scale"), score_bias=gctl.get("score_bias"), log_alphas=gla,
                    etas=geta)
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
    if "score_bias" in octl:
        spec_dict["score_bias"] = octl["score_bias"]
    want = omixer.kernel_core(oq, ok_, ov, oW1, oW2, spec_dict, log_alphas=ola, etas=oeta, mode=mode,
                              read_norm=READ.get(name, "key_mass"), eps=EPS.get(name, 1e-6), chunk=64)
    (want.transpose(1, 2) * w_out).sum().backward()

    assert rel_err(y, want.transpose(1, 2)) < BF16_TOL
    pairs = [("q", gq, oq), ("k", gk, ok_), ("v", gv, ov), ("W1", gW1, oW1), ("W2", gW2, oW2)]
    pairs += [(key, gctl[key], octl[key]) for key in ctl]
    if las is not None:
        pairs += [("eta", geta, oeta)]
        if name not in ILL_CONDITIONED_RETENTION | OPEN_PRECISION_RETENTION:
            pairs += [("log_alpha", gla, ola)]
    for label, got, ref in pairs:
        assert rel_err(got.grad, ref.grad) < BF16_TOL, label


def test_stale_bank_sequence_shards_are_rejected(dev):
    """Stale scans take no boundary states, so a sharded stale bank must raise
    rather than drop the earlier shards' memory."""
    from thetascan_b200.kernel import KernelSpec, kernel_core_sharded
    from thetascan_b200.seqpar import SeqShard
    qkv = torch.zeros(1, 8, 3 * 2 * 64, dtype=torch.bfloat16, device=dev)
    W1 = torch.zeros(2, 64, 64, device=dev)
    with pytest.raises(NotImplementedError):
        kernel_core_sharded(qkv, 2, W1, W1, KernelSpec(kind="softmax_partition", mode="stale"), None,
                            SeqShard(0, 1, lambda u: [u]), log_alphas=torch.zeros(1, 2, device=dev),
                            etas=torch.zeros(1, 2, device=dev))


PROLOGUE_CASES = {
    # name: (kind, P, basis, mode, J, B, H, T, d, rot)
    "relu2_partial_rope": ("relu2_ridge", 256, 1, "fast", 1, 2, 2, 300, 64, 32),
    "softmax_d40_rope20": ("softmax_partition", 64, 1, "sum", 0, 1, 3, 129, 40, 20),
    "bspline_full_rope": ("projected_bspline", 8, 16, "fast", 2, 1, 2, 200, 64, 64),
    "relu2_norm_only": ("relu2_ridge", 128, 1, "sum", 0, 2, 1, 77, 64, 0),
}


@pytest.mark.parametrize("name", list(PROLOGUE_CASES))
def test_fused_prologue_matches_torch_prologue(dev, name):
    """RoPE + L2 norm inside the feature kernels (``kernel_core_qkv``) against
    the same transforms as f32 PyTorch ops in front of ``kernel_core``: output,
    d qkv (all three slots) and the weight gradients.  Both run bf16 streams;
    they differ by one bf16 rounding of the q/k gradient (the unfused chain
    rounds it before the norm backward) and the order of the norm's sum."""
    from thetascan_b200.kernel import KernelSpec, Prologue, kernel_core, kernel_core_qkv
    from thetascan_b200.mixer import _rope, _rope_tables

    kind, P, basis, mode, J, B, H, T, d, rot = PROLOGUE_CASES[name]
    g = torch.Generator().manual_seed(sum(map(ord, name)))
    qkv = (torch.randn(B, T, 3 * H * d, generator=g) * 0.7).to(torch.bfloat16)
    m = P * basis
    W1 = torch.randn(H, P, d, generator=g) / math.sqrt(d)
    W2 = torch.randn(H, d, m, generator=g) * 0.2
    thr = torch.randn(H, generator=g) * 0.1 if kind == "relu2_ridge" else None
    gain = 4.0 + 8.0 * torch.rand(H, generator=g) if kind == "softmax_partition" else None
    scale = 0.5 + torch.rand(H, generator=g) if kind == "projected_bspline" else None
    las = etas = None
    if J:
        las = (0.9 + 0.099 * torch.rand(J, H, generator=g)).log()
        etas = torch.randn(J, H, generator=g) * 0.5
    w_out = torch.randn(B, T, H, d, generator=g).to(dev)
    spec = KernelSpec(kind=kind, mode=mode, basis=basis)

    def leaves():
        return [None if x is None else x.to(dev).clone().requires_grad_(True)
                for x in (qkv, W1, W2, thr, gain, scale, las, etas)]

    def ctl(t, gn, sc):
        return dict(threshold=t, gain=gn, spline_scale=sc)

    # fused
    a = leaves()
    cos = sin = None
    if rot:
        cos, sin = _rope_tables(T, rot, 10000.0, str(dev))
    y_f = kernel_core_qkv(a[0], H, a[1], a[2], spec, Prologue(rot, cos, sin, 1e-6), log_alphas=a[6],
                          etas=a[7], **ctl(a[3], a[4], a[5]))
    (y_f.float() * w_out).sum().backward()

    # unfused: torch prologue in f32, then the plain entry point
    b = leaves()
    q, k, v = b[0].view(B, T, 3, H, d).permute(2, 0, 3, 1, 4)

    def prep(x):
        x = _rope(x.float(), rot, 10000.0)
        return (x / x.norm(dim=-1, keepdim=True).clamp_min(1e-6)).to(torch.bfloat16).contiguous()

    y_u = kernel_core(prep(q), prep(k), v.contiguous(), b[1], b[2], spec, log_alphas=b[6], etas=b[7],
                      **ctl(b[3], b[4], b[5]))
    (y_u.float() * w_out).sum().backward()

    assert rel_err(y_f, y_u) < 1e-2
    dq_f, dk_f, dv_f = a[0].grad.view(B, T, 3, H, d).unbind(2)
    dq_u, dk_u, dv_u = b[0].grad.view(B, T, 3, H, d).unbind(2)
    for label, got, want in (("dq", dq_f, dq_u), ("dk", dk_f, dk_u), ("dv", dv_f, dv_u),
                             ("W1", a[1].grad, b[1].grad), ("W2", a[2].grad, b[2].grad)):
        assert rel_err(got, want) < 1e-2, label
    for i in range(3, 8):
        if a[i] is not None:
            assert rel_err(a[i].grad, b[i].grad) < 1e-2, i
