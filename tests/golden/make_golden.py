"""Generate golden fixtures from the reference ThetaScan package.

Run in the build container, where the reference project is importable:

    PYTHONPATH=<reference>/src python tests/golden/make_golden.py <out_dir>

It writes ``scan_cases.pt``, ``feature_cases.pt`` and ``mixer_cases.pt`` into
``<out_dir>`` (default: this directory).  Everything is computed by the
reference's own public module and core ops in float64 with fixed seeds, so the
fixtures pin both the CPU oracle (``oracle/``) and the CUDA path.  The GPU box
never runs this script; it only reads the fixtures.
"""
from __future__ import annotations

import math
import os
import sys

import torch


def _seeded(seed, *shape, dtype=torch.float64):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g, dtype=dtype)


def scan_cases():
    from thetascan._core.ops import scan_chunk, scan_cumsum, scan_naive

    cases = []
    B, H, T, Dk, Dv = 2, 3, 37, 5, 4
    q, k, v = (_seeded(s, B, H, T, d) for s, d in ((1, Dk), (2, Dk), (3, Dv)))
    log_alpha = torch.tensor([-0.05, -0.4, -2.0], dtype=torch.float64)
    stream = -_seeded(4, B, H, T, 1).abs() * 0.3
    for name, retention in (("sum", None), ("static", log_alpha), ("stream", stream)):
        leaves = [x.clone().requires_grad_(True) for x in (q, k, v)]
        ret = None if retention is None else retention.clone().requires_grad_(True)
        if retention is None:
            out = scan_chunk.linattn(*leaves, chunk=8)
        elif retention.ndim == 1:
            out = scan_chunk.linattn(*leaves, chunk=8, log_alpha=ret)
        else:
            out = scan_chunk.linattn(*leaves, ret, chunk=8)
        out.square().sum().backward()
        naive = scan_naive.linattn(q, k, v, None if retention is None else (
            retention.view(1, H, 1, 1).expand(B, H, T, 1) if retention.ndim == 1 else retention))
        cases.append({
            "name": name, "q": q, "k": k, "v": v, "retention": retention, "chunk": 8,
            "out": out.detach(), "naive": naive,
            "grads": [x.grad for x in leaves] + [None if ret is None else ret.grad],
        })
    cumsum = scan_cumsum.linattn(q, k, v)
    views = scan_chunk.linattn_views(q, k, v, (None, log_alpha, log_alpha * 3.0), chunk=16)
    return {"cases": cases, "cumsum_sum": cumsum, "views": views,
            "views_inputs": (q, k, v, log_alpha)}


def feature_cases():
    from thetascan._core.ops import kernel_features as kf

    pre = _seeded(10, 2, 3, 17, 16)
    thr = torch.tensor([0.0, 0.3, -0.2], dtype=torch.float64)
    bias = _seeded(11, 3, 16) * 0.1
    gain = torch.tensor([8.0, 4.0, 12.0], dtype=torch.float64)
    spline_pre = _seeded(12, 2, 3, 17, 4) * 2.0
    edge = torch.tensor([-3.5, -3.0, -1.0, 0.0, 1e-9, 1.0, 2.999, 3.0, 7.0], dtype=torch.float64)
    return {
        "pre": pre, "thr": thr, "bias": bias, "gain": gain, "spline_pre": spline_pre, "edge": edge,
        "relu2": kf.relu2_ridge_features(pre, score_bias=None, relu2_threshold=thr, eps=1e-6),
        "relu2_bias": kf.relu2_ridge_features(pre, score_bias=bias, eps=1e-6),
        "relu2_dead": kf.relu2_ridge_features(-pre.abs() - 1.0, score_bias=None, eps=1e-6),
        "softmax": kf.softmax_partition_features(
            pre, gain=gain, fallback_gain=8.0, score_bias=bias, sparsity="none",
            relative_threshold=None, threshold_temperature=0.25, eps=1e-6),
        "bspline": kf.projected_bspline_features(
            spline_pre, n_basis=8, degree=3, bound=3.0, scale=None, fallback_scale=1.0),
        "bspline16": kf.projected_bspline_features(
            spline_pre, n_basis=16, degree=3, bound=3.0, scale=None, fallback_scale=1.0),
        "bspline_edge": kf.open_uniform_bspline_basis(edge, n_basis=8, degree=3, bound=3.0),
    }


MIXER_CONFIGS = {
    # Config-1 family at a fixture-sized shape: softmax partition, bank (fast).
    "softmax_bank_fast": dict(
        d_model=64, n_heads=2, memory_multiplier=1, family="kernel",
        kernel=dict(feature_map="softmax_partition"),
        temporal=dict(mode="bank", retention_init=0.95), B=2, T=40),
    # Config-2 family: relu2 ridge, 2x expansion, partial RoPE, bank.
    "relu2_expanded_rope": dict(
        d_model=64, n_heads=2, memory_multiplier=4, feature_expansion=2, family="kernel",
        kernel=dict(feature_map="relu2_ridge", relu2_threshold_mode="learned_per_head"),
        rope=dict(mode="partial", fraction=0.5), temporal=dict(mode="bank", recency_branches=2,
                                                               retention_inits=(0.9, 0.99)),
        B=2, T=40),
    # Config-4 family: projected B-spline with a stale bank.
    "bspline_stale": dict(
        d_model=64, n_heads=2, memory_multiplier=2, family="kernel",
        kernel=dict(feature_map="projected_bspline", bspline_basis_count=16),
        temporal=dict(mode="bank", bank_mode="stale", retention_init=0.9), B=2, T=40),
    # Plain sum with per-feature mass normalization.
    "softmax_sum_feature_mass": dict(
        d_model=64, n_heads=2, memory_multiplier=1, family="kernel",
        kernel=dict(feature_map="softmax_partition", read_normalization="feature_mass"),
        B=2, T=40),
    # Kernel-tile-shaped case (head_dim 64, ragged T) for the CUDA path.
    "relu2_d64_ragged": dict(
        d_model=128, n_heads=2, memory_multiplier=2, family="kernel",
        kernel=dict(feature_map="relu2_ridge"),
        rope=dict(mode="partial", fraction=0.5), temporal=dict(mode="bank", retention_init=0.9),
        B=1, T=160, dtype="float32"),
    # The same shape with a stale bank (the zero-memory base read in the blend).
    "gn_d64_stale": dict(
        d_model=128, n_heads=2, memory_multiplier=2, share_key_query=True, output_gate=False, family="gn",
        gn=dict(nonlinearity="relu2", read_normalization="both_feature_mass"),
        rope=dict(mode="partial", fraction=0.5),
        temporal=dict(mode="bank", bank_mode="stale", retention_init=0.9), B=1, T=160, dtype="float32"),
}


def mixer_cases():
    from thetascan import (KernelConfig, RoPEConfig, TemporalConfig, ThetaScan,
                           ThetaScanConfig)

    out = {}
    for name, spec in MIXER_CONFIGS.items():
        spec = dict(spec)
        B, T = spec.pop("B"), spec.pop("T")
        dtype = getattr(torch, spec.pop("dtype", "float64"))
        kernel = KernelConfig(**spec.pop("kernel", {}))
        rope = RoPEConfig(**spec.pop("rope", {}))
        temporal = TemporalConfig(**spec.pop("temporal", {}))
        cfg = ThetaScanConfig(kernel=kernel, rope=rope, temporal=temporal, **spec)
        torch.manual_seed(0)
        module = ThetaScan(cfg).to(torch.float64)
        core = module._core
        # Nonzero W2 and blends so every branch of the read carries gradient.
        with torch.no_grad():
            for p in core.W2:
                p.copy_(_seeded(5, *p.shape) * 0.2)
            if core.fade_eta is not None:
                core.fade_eta.copy_(_seeded(6, *core.fade_eta.shape) * 0.5)
            if getattr(core, "kernel_relu2_threshold", None) is not None:
                core.kernel_relu2_threshold.copy_(_seeded(7, *core.kernel_relu2_threshold.shape) * 0.1)
        x = _seeded(8, B, T, cfg.d_model).requires_grad_(True)
        y = module(x)
        weight = _seeded(9, *y.shape)
        (y * weight).sum().backward()
        params = {n: t.detach().to(dtype) for n, t in core.state_dict(keep_vars=True).items()
                  if t is not None}
        for n, buf in core.named_buffers():
            if buf is not None and n not in params:
                params[n] = buf.detach().to(dtype)
        grads = {n: p.grad.detach().to(dtype) for n, p in core.named_parameters() if p.grad is not None}
        core_cfg = module._core_config
        out[name] = {
            "public_config": cfg.to_dict(), "B": B, "T": T,
            "core": {k: getattr(core_cfg, k) for k in (
                "d_model", "n_heads", "head_dim", "mem_hidden", "feature_expansion", "expansion_key",
                "kernel_kind", "softmax_gain", "bspline_basis_count", "bspline_bound", "bspline_scale",
                "rope", "rope_frac", "rope_base", "read_fade", "read_fade_mode", "fade_blend_mode",
                "read_norm", "read_norm_mode", "eps", "scan_chunk", "share_kq", "key_value_heads")},
            "params": params, "x": x.detach().to(dtype), "y": y.detach().to(dtype),
            "out_weight": weight.to(dtype), "x_grad": x.grad.detach().to(dtype), "grads": grads,
        }
    return out


GN_CONFIGS = {
    # Config-3 parity family: relu2, two-stage normalized read, one fast branch,
    # shared k/q projection (the gn_reference_v0_1 preset at fixture size).
    "gn_both_relu2_bank": dict(
        d_model=64, n_heads=2, memory_multiplier=3, share_key_query=True, output_gate=False, family="gn",
        gn=dict(nonlinearity="relu2", read_normalization="both_feature_mass"),
        rope=dict(mode="partial", fraction=0.5), temporal=dict(mode="bank", retention_init=0.9), B=2, T=40),
    # gn_expanded_reference_v0_1 at fixture size: learned threshold, 2x expansion.
    "gn_both_threshold_expanded": dict(
        d_model=64, n_heads=2, memory_multiplier=6, feature_expansion=2, share_key_query=True,
        output_gate=False, family="gn",
        gn=dict(nonlinearity="relu2_threshold", read_normalization="both_feature_mass"),
        rope=dict(mode="partial", fraction=0.5), temporal=dict(mode="bank", retention_init=0.9), B=2, T=40),
    # Normalized W2 read only, plain sum, output gate, per-head projections.
    "gn_w2_relu2_sum": dict(
        d_model=64, n_heads=2, memory_multiplier=2, family="gn",
        gn=dict(nonlinearity="relu2", read_normalization="w2_feature_mass"), B=2, T=40),
    # Unnormalized read with silu and a two-branch fast bank.
    "gn_none_silu_bank2": dict(
        d_model=64, n_heads=2, memory_multiplier=2, family="gn",
        gn=dict(nonlinearity="silu", read_normalization="none"),
        temporal=dict(mode="bank", recency_branches=2, retention_inits=(0.9, 0.99)), B=2, T=40),
    # Kernel-tile-shaped case for the CUDA path (head_dim 64, m = 128, ragged T).
    "gn_d64_ragged": dict(
        d_model=128, n_heads=2, memory_multiplier=2, share_key_query=True, output_gate=False, family="gn",
        gn=dict(nonlinearity="relu2", read_normalization="both_feature_mass"),
        rope=dict(mode="partial", fraction=0.5), temporal=dict(mode="bank", retention_init=0.9),
        B=1, T=160, dtype="float32"),
    # The same shape with a stale bank (the zero-memory base read in the blend).
    "gn_d64_stale": dict(
        d_model=128, n_heads=2, memory_multiplier=2, share_key_query=True, output_gate=False, family="gn",
        gn=dict(nonlinearity="relu2", read_normalization="both_feature_mass"),
        rope=dict(mode="partial", fraction=0.5),
        temporal=dict(mode="bank", bank_mode="stale", retention_init=0.9), B=1, T=160, dtype="float32"),
}

# Two Jacobian steps (write_iters == 2, engine.py:323-339): unnormalized
# reads (the reference requires it), a fast bank, head_dim 64, ragged T;
# one relu2 and one silu net with a learned threshold alternative.
GN_JAC2_CONFIGS = {
    "gn_jac2_relu2_bank": dict(
        d_model=128, n_heads=2, memory_multiplier=2, family="gn",
        gn=dict(nonlinearity="relu2", jacobian_steps=2, read_normalization="none"),
        rope=dict(mode="partial", fraction=0.5), temporal=dict(mode="bank", retention_init=0.9),
        B=1, T=160, dtype="float32"),
    "gn_jac2_threshold_sum": dict(
        d_model=128, n_heads=2, memory_multiplier=2, share_key_query=True, output_gate=False, family="gn",
        gn=dict(nonlinearity="relu2_threshold", jacobian_steps=2, read_normalization="none"),
        rope=dict(mode="partial", fraction=0.5), B=2, T=96, dtype="float32"),
}

# GN nets the one-block row kernels do not cover: the swiglu activation and
# depth > 1 (engine.py:117-175, 215-255), with one and two Jacobian steps,
# each read normalisation and fast / stale banks; head_dim 64, ragged T.
GN_DEEP_CONFIGS = {
    "gn_swiglu_sum": dict(
        d_model=128, n_heads=2, memory_multiplier=2, family="gn",
        gn=dict(nonlinearity="swiglu", read_normalization="none"),
        rope=dict(mode="partial", fraction=0.5), B=2, T=96, dtype="float32"),
    "gn_swiglu_jac2_bank": dict(
        d_model=128, n_heads=2, memory_multiplier=2, share_key_query=True, output_gate=False, family="gn",
        gn=dict(nonlinearity="swiglu", jacobian_steps=2, read_normalization="none"),
        rope=dict(mode="partial", fraction=0.5), temporal=dict(mode="bank", retention_init=0.9),
        B=1, T=160, dtype="float32"),
    "gn_depth2_both_bank": dict(
        d_model=128, n_heads=2, memory_multiplier=2, depth=2, share_key_query=True, output_gate=False,
        family="gn", gn=dict(nonlinearity="relu2", read_normalization="both_feature_mass"),
        rope=dict(mode="partial", fraction=0.5), temporal=dict(mode="bank", retention_init=0.9),
        B=1, T=160, dtype="float32"),
    "gn_depth2_swiglu_stale": dict(
        d_model=128, n_heads=2, memory_multiplier=2, depth=2, family="gn",
        gn=dict(nonlinearity="swiglu", read_normalization="none"),
        temporal=dict(mode="bank", bank_mode="stale", retention_init=0.9), B=1, T=128, dtype="float32"),
    "gn_depth3_threshold_w2_expanded": dict(
        d_model=128, n_heads=2, memory_multiplier=2, feature_expansion=2, depth=3, family="gn",
        gn=dict(nonlinearity="relu2_threshold", read_normalization="w2_feature_mass"),
        rope=dict(mode="partial", fraction=0.5), B=2, T=96, dtype="float32"),
    "gn_depth2_silu_jac2_bank2": dict(
        d_model=128, n_heads=2, memory_multiplier=2, depth=2, family="gn",
        gn=dict(nonlinearity="silu", jacobian_steps=2, read_normalization="none"),
        temporal=dict(mode="bank", recency_branches=2, retention_inits=(0.9, 0.99)),
        B=1, T=128, dtype="float32"),
}

# Config-3 width (head_dim 128, m = 128, relu2, two-stage feature-mass read,
# the plain sum view) at T = 1024; written to its own file, gn_c3_cases.pt.
GN_C3_CONFIGS = {
    "gn_c3_d128_T1024": dict(
        d_model=256, n_heads=2, memory_multiplier=1, family="gn",
        gn=dict(nonlinearity="relu2", read_normalization="both_feature_mass"),
        rope=dict(mode="partial", fraction=0.5), temporal=dict(mode="sum"), B=1, T=1024, dtype="float32"),
}

GN_CORE_KEYS = (
    "d_model", "n_heads", "head_dim", "mem_hidden", "feature_expansion", "expansion_key", "depth",
    "write_rule", "nonlin", "learn_thresh", "write_iters", "fast_w1", "act_norm", "qk_norm",
    "rope", "rope_frac", "rope_base", "read_fade", "read_fade_mode", "fade_blend_mode",
    "read_norm", "read_norm_w1", "read_norm_mode", "eps", "scan_chunk", "share_kq", "key_value_heads")


def gn_cases(configs=None):
    from thetascan import GNConfig, RoPEConfig, TemporalConfig, ThetaScan, ThetaScanConfig

    out = {}
    for name, spec in (GN_CONFIGS if configs is None else configs).items():
        spec = dict(spec)
        B, T = spec.pop("B"), spec.pop("T")
        dtype = getattr(torch, spec.pop("dtype", "float64"))
        gn = GNConfig(**spec.pop("gn", {}))
        rope = RoPEConfig(**spec.pop("rope", {}))
        temporal = TemporalConfig(**spec.pop("temporal", {}))
        cfg = ThetaScanConfig(gn=gn, rope=rope, temporal=temporal, **spec)
        torch.manual_seed(0)
        module = ThetaScan(cfg).to(torch.float64)
        core = module._core
        with torch.no_grad():
            for p in core.W2:
                p.copy_(_seeded(5, *p.shape) * 0.2)
            if core.fade_eta is not None:
                core.fade_eta.copy_(_seeded(6, *core.fade_eta.shape) * 0.5)
            if core.Wg is not None:
                for p in core.Wg:
                    p.copy_(_seeded(7, *p.shape) * 0.1)
            if getattr(core, "kq_bias", None) is not None:
                core.kq_bias.copy_(_seeded(10, *core.kq_bias.shape) * 0.1)
        x = _seeded(8, B, T, cfg.d_model).requires_grad_(True)
        y = module(x)
        weight = _seeded(9, *y.shape)
        (y * weight).sum().backward()
        params = {n: t.detach().to(dtype) for n, t in core.state_dict(keep_vars=True).items()
                  if t is not None}
        for n, buf in core.named_buffers():
            if buf is not None and n not in params:
                params[n] = buf.detach().to(dtype)
        grads = {n: p.grad.detach().to(dtype) for n, p in core.named_parameters() if p.grad is not None}
        core_cfg = module._core_config
        out[name] = {
            "public_config": cfg.to_dict(), "B": B, "T": T,
            "core": {k: getattr(core_cfg, k) for k in GN_CORE_KEYS},
            "params": params, "x": x.detach().to(dtype), "y": y.detach().to(dtype),
            "out_weight": weight.to(dtype), "x_grad": x.grad.detach().to(dtype), "grads": grads,
        }
    return out


def gn_c3_cases():
    return gn_cases(GN_C3_CONFIGS)


def gn_tanh_cases():
    """Config 3 as the baseline states it -- a tanh GN net with damping 1e-2 --
    which the reference's configuration cannot express: its GN nonlinearity
    table (nonlin.py:28-31) has no tanh and its public config no damping.  The
    fixture runs the reference's own engine with the table extended by
    (tanh, 1 - h^2) and the core epsilon (_core/config.py:191: the damping of
    the lambda solve, engine.py:255, and the L2/RMS/read epsilons) set to
    1e-2 on the constructed module; the read is unnormalized, since the
    feature-mass normalizations need nonnegative features
    (_core/config.py:420-423).  Head dim 128, m = 128, the plain sum view
    and a two-branch fast bank.  The matching b200 config is stored beside."""
    from thetascan import GNConfig, RoPEConfig, TemporalConfig, ThetaScan, ThetaScanConfig
    from thetascan._core.ops import nonlin

    nonlin.ELEMENTWISE.setdefault("tanh", (torch.tanh, lambda pre, h: 1.0 - h * h))
    out = {}
    specs = {
        "gn_tanh_d128_sum": (TemporalConfig(mode="sum"), 1, 256),
        "gn_tanh_d128_bank2": (TemporalConfig(mode="bank", recency_branches=2, retention_inits=(0.9, 0.99)), 1, 200),
    }
    for name, (temporal, B, T) in specs.items():
        cfg = ThetaScanConfig(d_model=256, n_heads=2, memory_multiplier=1, family="gn",
                              gn=GNConfig(nonlinearity="relu2", read_normalization="none"),
                              rope=RoPEConfig(mode="partial", fraction=0.5), temporal=temporal)
        torch.manual_seed(0)
        module = ThetaScan(cfg).to(torch.float64)
        core = module._core
        core.cfg.nonlin = "tanh"
        core.cfg.eps = 1e-2
        with torch.no_grad():
            for p in core.W2:
                p.copy_(_seeded(5, *p.shape) * 0.2)
            if core.fade_eta is not None:
                core.fade_eta.copy_(_seeded(6, *core.fade_eta.shape) * 0.5)
        x = _seeded(8, B, T, cfg.d_model).requires_grad_(True)
        y = module(x)
        weight = _seeded(9, *y.shape)
        (y * weight).sum().backward()
        b200_cfg = cfg.to_dict()
        b200_cfg["gn"] = dict(b200_cfg["gn"], nonlinearity="tanh", damping=1e-2)
        out[name] = {
            "public_config": cfg.to_dict(), "b200_config": b200_cfg, "B": B, "T": T,
            "core": {k: getattr(core.cfg, k) for k in GN_CORE_KEYS},
            "params": {n: t.detach().float() for n, t in core.state_dict(keep_vars=True).items() if t is not None},
            "x": x.detach().float(), "y": y.detach().float(), "out_weight": weight.float(),
            "x_grad": x.grad.detach().float(),
            "grads": {n: p.grad.detach().float() for n, p in core.named_parameters() if p.grad is not None},
        }
    return out


# Relative sparsity of the softmax partition (kernel_features.py:43-113),
# head_dim 64 and m = 128 (the kernel-tile shape), fast bank, ragged T.
SPARSE_MIXERS = {
    f"softmax_{mode}": dict(
        d_model=128, n_heads=2, memory_multiplier=2, family="kernel",
        kernel=dict(feature_map="softmax_partition", sparsity=mode,
                    sparse_blend_init=0.5 if mode == "relative_st_blend" else 0.0),
        rope=dict(mode="partial", fraction=0.5), temporal=dict(mode="bank", retention_init=0.9),
        B=1, T=160, dtype="float32")
    for mode in ("relative_soft", "relative_st", "relative_st_blend")
}


def sparse_cases():
    """Feature-level cases (the map, its gradient to the scores, the cutoff
    and the blend) and whole mixers with each sparsity mode, from the
    reference itself."""
    from thetascan import KernelConfig, RoPEConfig, TemporalConfig, ThetaScan, ThetaScanConfig
    from thetascan._core.ops import kernel_features as kf

    out = {"features": {}, "mixers": {}}
    pre = _seeded(20, 2, 3, 17, 16) * 0.5
    bias = _seeded(21, 3, 16) * 0.1
    gain = torch.tensor([8.0, 4.0, 12.0], dtype=torch.float64)
    weight = _seeded(22, 2, 3, 17, 16)
    for mode in ("relative_soft", "relative_st", "relative_st_blend"):
        p = pre.clone().requires_grad_(True)
        rho = torch.tensor([0.05, 0.2, 0.01], dtype=torch.float64, requires_grad=True)
        alpha = torch.tensor([0.3, 0.7, 1.0], dtype=torch.float64, requires_grad=True)
        phi = kf.softmax_partition_features(
            p, gain=gain, fallback_gain=8.0, score_bias=bias, sparsity=mode, relative_threshold=rho,
            sparse_blend_alpha=alpha if mode == "relative_st_blend" else None, threshold_temperature=0.25,
            eps=1e-6)
        (phi * weight).sum().backward()
        out["features"][mode] = {
            "pre": pre, "bias": bias, "gain": gain, "rho": rho.detach(), "alpha": alpha.detach(),
            "weight": weight, "phi": phi.detach(), "dpre": p.grad, "drho": rho.grad,
            "dalpha": None if alpha.grad is None else alpha.grad}
    for name, spec in SPARSE_MIXERS.items():
        spec = dict(spec)
        B, T = spec.pop("B"), spec.pop("T")
        dtype = getattr(torch, spec.pop("dtype"))
        cfg = ThetaScanConfig(kernel=KernelConfig(**spec.pop("kernel")), rope=RoPEConfig(**spec.pop("rope")),
                              temporal=TemporalConfig(**spec.pop("temporal")), **spec)
        torch.manual_seed(0)
        module = ThetaScan(cfg).to(torch.float64)
        core = module._core
        with torch.no_grad():
            for p in core.W2:
                p.copy_(_seeded(5, *p.shape) * 0.2)
            if core.fade_eta is not None:
                core.fade_eta.copy_(_seeded(6, *core.fade_eta.shape) * 0.5)
            # a cutoff that removes a visible share of the features
            core.kernel_relative_threshold_raw.copy_(torch.tensor([-2.0, -3.0], dtype=torch.float64))
            # float32-representable inputs: the stored fixture is exact for
            # them (a hard gate would flip under a later rounding)
            for p in module.parameters():
                p.copy_(p.to(dtype).to(torch.float64))
        x = _seeded(8, B, T, cfg.d_model).to(dtype).to(torch.float64).requires_grad_(True)
        y = module(x)
        w = _seeded(9, *y.shape)
        (y * w).sum().backward()
        core_cfg = module._core_config
        out["mixers"][name] = {
            "public_config": cfg.to_dict(), "B": B, "T": T,
            "core": {k: getattr(core_cfg, k) for k in (
                "d_model", "n_heads", "head_dim", "mem_hidden", "feature_expansion", "expansion_key",
                "kernel_kind", "softmax_gain", "bspline_basis_count", "bspline_bound", "bspline_scale",
                "rope", "rope_frac", "rope_base", "read_fade", "read_fade_mode", "fade_blend_mode",
                "read_norm", "read_norm_mode", "eps", "scan_chunk", "share_kq", "key_value_heads",
                "kernel_sparsity", "kernel_threshold_temperature")},
            "params": {n: t.detach().to(dtype) for n, t in core.state_dict(keep_vars=True).items()
                       if t is not None},
            "x": x.detach().to(dtype), "y": y.detach().to(dtype), "out_weight": w.to(dtype),
            "x_grad": x.grad.detach().to(dtype),
            "grads": {n: p.grad.detach().to(dtype) for n, p in core.named_parameters() if p.grad is not None},
        }
    return out


def gn_jac2_cases():
    return gn_cases(GN_JAC2_CONFIGS)


def gn_deep_cases():
    return gn_cases(GN_DEEP_CONFIGS)


GENERATORS = {"scan": scan_cases, "feature": feature_cases, "mixer": mixer_cases, "gn": gn_cases,
              "gn_jac2": gn_jac2_cases, "gn_deep": gn_deep_cases,
              "gn_c3": gn_c3_cases, "gn_tanh": gn_tanh_cases, "sparse": sparse_cases}


def main():
    # usage: make_golden.py [out_dir] [scan,feature,mixer,gn]
    target = sys.argv[1] if len(sys.argv) > 1 else os.path.dirname(os.path.abspath(__file__))
    which = sys.argv[2].split(",") if len(sys.argv) > 2 else list(GENERATORS)
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    for name in which:
        torch.save(GENERATORS[name](), os.path.join(target, f"{name}_cases.pt"))
    print("golden fixtures written to", target, which)


if __name__ == "__main__":
    main()
