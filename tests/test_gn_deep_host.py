"""Host algebra of the deep / swiglu GN core (``thetascan_b200.gn_deep``) on CPU.

The core's per-token maps are PyTorch; its sequence reads go through the
float32 scan kernels.  Here the scan is replaced by the float64 oracle scan (the
checker, injected by the test only), so that the write, the per-layer reads,
the view grouping and the bank blend are pinned on CPU against fixtures of
the reference GN mixer itself (``tests/golden/gn_deep_cases.pt``): output,
input gradient and every parameter gradient, float32 per-token maps, at
``1e-4`` of each quantity's largest entry.
"""
from __future__ import annotations

import os
import types

import pytest
import torch
import torch.nn.functional as F

from oracle import scan as oracle_scan
from thetascan_b200 import gn_deep, seqpar
from thetascan_b200.config import ThetaScanConfig
from thetascan_b200.mixer import ThetaScan, _l2, _rope

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
CASES = ["gn_swiglu_sum", "gn_swiglu_jac2_bank", "gn_depth2_both_bank", "gn_depth2_swiglu_stale",
         "gn_depth3_threshold_w2_expanded", "gn_depth2_silu_jac2_bank2"]
TOL = 1e-4


def rel_err(got, want):
    got, want = got.detach().double(), want.detach().double()
    return float((got - want).abs().max() / want.abs().max().clamp_min(1e-30))


def oracle_views(q, k, v, retentions, chunk=512, *, append_unit=False, stale=None):
    """float64 CPU stand-in for ``scan.linattn_views`` (same arguments and
    results: reads of every retention in the stream dtype, ``[v | 1]`` with
    ``append_unit``, the stale view as the plain sum minus the decayed
    read)."""
    stale = stale or (False,) * len(retentions)
    if append_unit:
        v = torch.cat([v, v.new_ones(*v.shape[:3], 1)], dim=-1)
    rets = tuple(None if r is None else r.double() for r in retentions) + (None,)
    outs = oracle_scan.linattn_chunk_views(q.double(), k.double(), v.double(), rets, 64)
    return tuple((outs[-1] - o if st else o).to(q.dtype) for o, st in zip(outs[:-1], stale))


def _mixer(core, cfg, x, shard=None):
    """The GN mixer's forward around ``gn_deep._core`` (float32 projections,
    RoPE from the shard's first position, L2 norm, gate, out projection)."""
    gn = cfg.gn
    B, T, _ = x.shape
    H, d = core.n_heads, core.head_dim
    pos0 = 0 if shard is None else shard.rank * T
    q, k, v = core.project(x)
    q, k = _l2(_rope(q, core._rot, cfg.rope.base, pos0)), _l2(_rope(k, core._rot, cfg.rope.base, pos0))
    log_alphas, etas = core.fade()
    layers = [core.effective_weights(l) + (None if core.Wg is None else core.Wg[l],) for l in range(cfg.depth)]
    y = gn_deep._core(q, k, v.contiguous(), layers,
                      "relu2" if gn.nonlinearity == "relu2_threshold" else gn.nonlinearity,
                      gn.nonlinearity == "relu2_threshold", gn.read_normalization != "none",
                      gn.read_normalization == "both_feature_mass", log_alphas, etas,
                      core.spec.mode if log_alphas is not None else "sum", 1e-6, gn.jacobian_steps, shard)
    y = y.transpose(1, 2)
    if core.ogate is not None:
        lin = core.ogate.g.lin
        y = F.silu(F.linear(x, lin.weight, lin.bias)).view(B, T, H, d) * y
    return F.linear(y.reshape(B, T, H * d), core.proj_out.weight)


def run_case(case, monkeypatch, P=None):
    monkeypatch.setattr(gn_deep, "_scan", types.SimpleNamespace(linattn_views=oracle_views))
    cfg = ThetaScanConfig.from_dict(case["public_config"])
    module = ThetaScan(cfg)
    module.load_state_dict({"_core." + n: t.float() for n, t in case["params"].items()
                            if not n.startswith("_expand_")})
    x = case["x"].float().requires_grad_(True)
    if P is None:
        y = _mixer(module._core, cfg, x)
    else:
        runner = seqpar.SequentialShards(P)
        L = x.shape[1] // P
        y = torch.cat([_mixer(module._core, cfg, x[:, r * L:(r + 1) * L], runner.shard(r)) for r in range(P)],
                      dim=1)
    (y.double() * case["out_weight"]).sum().backward()
    return module, x, y


@pytest.mark.parametrize("name", CASES)
def test_gn_deep_algebra_matches_reference_fixture(name, monkeypatch):
    case = torch.load(os.path.join(GOLDEN, "gn_deep_cases.pt"), weights_only=False)[name]
    module, x, y = run_case(case, monkeypatch)
    assert rel_err(y, case["y"]) < TOL
    assert rel_err(x.grad, case["x_grad"]) < TOL
    grads = dict(module._core.named_parameters())
    assert set(case["grads"]) <= set(grads)
    for n, want in case["grads"].items():
        assert rel_err(grads[n].grad, want) < TOL, n


@pytest.mark.parametrize("name,P", [("gn_depth2_both_bank", 2), ("gn_depth2_swiglu_stale", 4),
                                    ("gn_swiglu_jac2_bank", 2)])
def test_gn_sequence_shards_match_reference_fixture(name, P, monkeypatch):
    """The GN family on P sequence shards run one after another
    (``SequentialShards``): every read of every layer enters with the earlier
    shards' state (``seqpar.sharded_reads``; both stages' streams are
    write-side), and the concatenated output and all gradients equal the
    reference's unsharded fixture."""
    case = torch.load(os.path.join(GOLDEN, "gn_deep_cases.pt"), weights_only=False)[name]
    module, x, y = run_case(case, monkeypatch, P)
    assert rel_err(y, case["y"]) < TOL
    assert rel_err(x.grad, case["x_grad"]) < TOL
    grads = dict(module._core.named_parameters())
    for n, want in case["grads"].items():
        assert rel_err(grads[n].grad, want) < TOL, n


@pytest.mark.parametrize("name", CASES)
def test_gn_deep_state_dict_and_seeded_init_match_reference(name):
    """Deep and swiglu GN modules: the reference's parameter names and shapes
    (per-layer W1 / W2 / Wg, the per-layer expansion maps), and with seed 0
    the same initial values for everything the fixture generator did not
    overwrite (W2, Wg, fade_eta, kq_bias)."""
    case = torch.load(os.path.join(GOLDEN, "gn_deep_cases.pt"), weights_only=False)[name]
    torch.manual_seed(0)
    module = ThetaScan(ThetaScanConfig.from_dict(case["public_config"]))
    ours = dict(module._core.state_dict())
    theirs = {n: t for n, t in case["params"].items() if not n.startswith("_expand_")}
    assert set(ours) == set(theirs)
    for n, t in ours.items():
        assert tuple(t.shape) == tuple(theirs[n].shape), n
        if not n.startswith(("W2.", "Wg.", "fade_eta", "kq_bias")):
            assert torch.equal(t.to(theirs[n].dtype), theirs[n]), n
    buffers = dict(module._core.named_buffers())
    for n, t in case["params"].items():
        if n.startswith("_expand_w"):
            assert torch.equal(buffers[n].to(t.dtype), t), n


def test_gn_deep_rejects_cpu_tensors():
    z = torch.zeros(1, 2, 8, 4)
    layers = [(torch.zeros(2, 8, 4), torch.zeros(2, 4, 8), None)]
    with pytest.raises(RuntimeError):
        gn_deep.gn_deep(z, z, z, layers)
