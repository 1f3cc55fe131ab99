"""The b200 mixer under ``torch.compile``: one graph, forward and backward.

The hot path is reached through ``torch.library`` custom ops with fake
implementations (``thetascan_b200.ops``), so Dynamo traces the whole mixer --
projections, RoPE, the fused core, gate, output projection -- into a single
graph with ``fullgraph=True, dynamic=False``, and a second and third step
reuse it instead of recompiling (the reference pins the same behaviour for
its chunk backend: tests/test_scan_chunk.py:663-738 of the reference
project).  The compiled step must also give the eager step's output.
"""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda")


def _configs():
    from thetascan_b200.config import KernelConfig, RoPEConfig, TemporalConfig, ThetaScanConfig
    fused = ThetaScanConfig(d_model=256, n_heads=4, memory_multiplier=4, feature_expansion=2, family="kernel",
                            kernel=KernelConfig(feature_map="relu2_ridge"),
                            rope=RoPEConfig(mode="partial", fraction=0.5),
                            temporal=TemporalConfig(mode="bank", retention_init=0.95))
    plain_sum = ThetaScanConfig(d_model=256, n_heads=4, memory_multiplier=2, family="kernel",
                                kernel=KernelConfig(feature_map="softmax_partition"),
                                temporal=TemporalConfig(mode="sum"))
    # the expanded kernel preset's layout (shared k/q projection with a per-head
    # bias, learned relu2 threshold, 2x expansion, two recency branches) at a
    # memory width the feature kernels take (m = 256)
    preset = ThetaScanConfig.from_dict({"preset": "kernel_expanded_reference_v0_1", "d_model": 128, "n_heads": 2})
    preset.memory_multiplier = 2
    return {"fused_qkv_bank": fused, "fused_qkv_sum": plain_sum, "shared_kq_preset": preset}


@pytest.mark.parametrize("name", ["fused_qkv_bank", "fused_qkv_sum", "shared_kq_preset"])
def test_mixer_traces_to_one_graph(dev, name):
    import torch._dynamo as dynamo
    from thetascan_b200.mixer import ThetaScan

    torch.manual_seed(11)
    module = ThetaScan(_configs()[name]).to(dev)
    with torch.no_grad():
        module._core.W2[0].normal_(0.0, 0.2)
        if module._core.fade_eta is not None:
            module._core.fade_eta.fill_(0.3)
    x = torch.randn(2, 200, module.config.d_model, device=dev).bfloat16()
    y_eager = module(x)
    dynamo.reset()
    dynamo.utils.counters.clear()
    compiled = torch.compile(module, backend="eager", fullgraph=True, dynamic=False)
    for _ in range(3):
        y = compiled(x)
        y.float().square().mean().backward()
        module.zero_grad(set_to_none=True)
    assert dynamo.utils.counters["stats"].get("unique_graphs", 0) == 1
    assert torch.equal(y, y_eager)


def test_compiled_gradients_match_eager(dev):
    from thetascan_b200.mixer import ThetaScan

    torch.manual_seed(12)
    module = ThetaScan(_configs()["fused_qkv_bank"]).to(dev)
    with torch.no_grad():
        module._core.W2[0].normal_(0.0, 0.2)
        module._core.fade_eta.fill_(0.3)
    x = torch.randn(2, 300, 256, device=dev).bfloat16()
    module(x).float().square().mean().backward()
    eager = {n: p.grad.clone() for n, p in module.named_parameters() if p.grad is not None}
    module.zero_grad(set_to_none=True)
    compiled = torch.compile(module, backend="eager", fullgraph=True, dynamic=False)
    compiled(x).float().square().mean().backward()
    for n, p in module.named_parameters():
        if n in eager:
            scale = eager[n].abs().max().clamp_min(1e-30)
            # same kernels; the weight gradients accumulate with atomics, so
            # their summation order may differ between runs
            assert float((p.grad - eager[n]).abs().max() / scale) < 1e-5, n


def test_scan_contract_traces_to_one_graph(dev):
    import torch._dynamo as dynamo
    from thetascan_b200 import scan

    g = torch.Generator(device="cpu").manual_seed(3)
    q = torch.randn(1, 2, 300, 64, generator=g).abs().to(dev).bfloat16().requires_grad_(True)
    k = torch.randn(1, 2, 300, 64, generator=g).abs().to(dev).bfloat16().requires_grad_(True)
    v = torch.randn(1, 2, 300, 64, generator=g).to(dev).bfloat16().requires_grad_(True)
    la = torch.log(torch.tensor([0.9, 0.99], device=dev)).requires_grad_(True)

    def views(q, k, v, la):
        a, b = scan.linattn_views(q, k, v, (None, la), 64)
        return (a.float() * b.float()).sum()

    dynamo.reset()
    dynamo.utils.counters.clear()
    compiled = torch.compile(views, backend="eager", fullgraph=True, dynamic=False)
    want = views(q, k, v, la)
    want.backward()
    grads = [t.grad.clone() for t in (q, k, v, la)]
    for t in (q, k, v, la):
        t.grad = None
    got = compiled(q, k, v, la)
    got.backward()
    assert dynamo.utils.counters["stats"].get("unique_graphs", 0) == 1
    assert torch.equal(got, want)
    for t, w in zip((q, k, v, la), grads):
        assert float((t.grad.float() - w.float()).abs().max() / w.float().abs().max()) < 1e-5
