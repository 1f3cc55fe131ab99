"""The hybrid LM host (config 5) with the b200 GN mixer against the same LM
with the reference package's own GN mixer (``tests/_refpkg.py``): the same
weights, the same tokens; loss and every parameter gradient.  Ours runs on
the GPU in float32 (the GN family's per-token math is float32, its scan
streams bf16); the reference runs in float64 on the CPU.  Tolerance 2e-2
(bf16 scan streams) on ``max|got - ref| / max|ref|``.
"""
from __future__ import annotations

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


def test_hybrid_lm_matches_lm_with_reference_mixer():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    ts = import_reference()
    from thetascan_b200.lm import HybridLM, gn_mixer_config

    def reference_mixer(cfg):
        d = cfg.to_dict()
        d["gn"] = {k: v for k, v in d["gn"].items() if k != "damping"}
        return ts.ThetaScan(ts.ThetaScanConfig.from_dict(d))

    kw = dict(vocab=256, d_model=128, n_layers=3, n_heads=2, mixer_layers=(1,),
              mixer_config=gn_mixer_config(128, 2))
    torch.manual_seed(5)
    ours = HybridLM(**kw)
    ref = HybridLM(**kw, mixer_factory=reference_mixer)
    ref.load_state_dict(ours.state_dict())
    with torch.no_grad():   # a nonzero mixer output so that its gradients flow
        for m in (ours, ref):
            m.blocks[1].mix._core.proj_out.weight.copy_(
                torch.randn(m.blocks[1].mix._core.proj_out.weight.shape, generator=torch.Generator().manual_seed(6))
                * 0.05)
    tokens = torch.randint(0, 256, (2, 201), generator=torch.Generator().manual_seed(7))
    ours = ours.cuda()
    loss = ours.loss(tokens.cuda())
    loss.backward()
    ref = ref.double()
    want = ref.loss(tokens)
    want.backward()
    assert abs(float(loss) - float(want)) / abs(float(want)) < 1e-3
    got = dict(ours.named_parameters())
    for name, p in ref.named_parameters():
        if p.grad is None:
            continue
        assert got[name].grad is not None, name
        assert rel_err(got[name].grad, p.grad) < 2e-2, name
