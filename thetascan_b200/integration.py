"""Register ``backend="b200"`` inside an installed reference ``thetascan``.

``install()`` patches a reference ThetaScan v0.1.0 package in place so that
``ThetaScanConfig(runtime=RuntimeConfig(backend="b200"))`` validates and runs
on this package's kernels, without forking the reference's math:

* the backend name is accepted where the reference lists its backends:
  the public validator (src/thetascan/config.py:458-463) and the core
  ``BACKENDS`` tuple (src/thetascan/_core/config.py:12);
* the scan-level plugin point routes ``"b200"`` to
  :func:`thetascan_b200.scan.linattn_views` -- ``interface._fn``
  (src/thetascan/_core/ops/interface.py:42-47) and the chunk branch of
  ``interface.scan_views`` (interface.py:175-182);
* the kernel-family mixer forward (src/thetascan/_core/modules/block.py:573-724)
  runs the fused hot path when the configuration is supported, by moving the
  module's parameters into a :class:`thetascan_b200.mixer.ThetaScanCore` view
  that shares their storage.

Everything stays CUDA-only: a ``"b200"`` module on a CPU tensor raises
``RuntimeError`` like the reference's FLA backend (scan_fla.py:57-58).
"""
from __future__ import annotations

import functools

_INSTALLED = False


def _scan_views_b200(q, k, v, retentions, chunk):
    from . import scan
    return scan.linattn_views(q, k, v, tuple(retentions), chunk)


def install():
    """Patch the importable reference ``thetascan`` package (idempotent)."""
    global _INSTALLED
    if _INSTALLED:
        return
    import thetascan.config as pub
    from thetascan._core import config as core
    from thetascan._core.modules import block
    from thetascan._core.ops import interface

    # 1. Backend name.
    if "b200" not in core.BACKENDS:
        core.BACKENDS = tuple(core.BACKENDS) + ("b200",)
    original_validate = pub.RuntimeConfig.validate

    @functools.wraps(original_validate)
    def validate(self):
        if self.backend == "b200":
            probe = pub.RuntimeConfig(backend="chunk", scan_chunk=self.scan_chunk)
            return original_validate(probe)
        return original_validate(self)

    pub.RuntimeConfig.validate = validate

    # 2. Scan-level plugin point.
    original_fn = interface._fn

    def _fn(backend, chunk=512):
        if backend == "b200":
            from . import scan
            return functools.partial(lambda q, k, v, decay=None, c=chunk: scan.linattn(q, k, v, decay, c))
        return original_fn(backend, chunk)

    interface._fn = _fn
    original_scan_views = interface.scan_views

    def scan_views(views, q, k, v, key_kind):
        terms = [view.scan_terms(key_kind) for view in views]
        contributing = next((view for view, t in zip(views, terms) if t), None)
        if contributing is None or contributing.backend != "b200":
            return original_scan_views(views, q, k, v, key_kind)
        # Same slot bookkeeping as the reference: one scan per distinct retention.
        retentions, slots = [], []
        for view_terms in terms:
            view_slots = []
            for _, retention in view_terms:
                slot = next((i for i, r in enumerate(retentions) if r is retention), None)
                if slot is None:
                    slot = len(retentions)
                    retentions.append(retention)
                view_slots.append(slot)
            slots.append(view_slots)
        chunk = getattr(contributing, "chunk", 512)
        scanned = _scan_views_b200(q, k, v, retentions, chunk)
        outputs = []
        for view_terms, view_slots in zip(terms, slots):
            if not view_terms:
                outputs.append(v.new_zeros(*q.shape[:3], v.shape[-1]))
                continue
            total = None
            for (coef, _), slot in zip(view_terms, view_slots):
                piece = scanned[slot] if coef == 1.0 else coef * scanned[slot]
                total = piece if total is None else total + piece
            outputs.append(total)
        return tuple(outputs)

    interface.scan_views = scan_views

    # 3. Fused mixer forward for supported kernel-family configurations.
    original_forward = block.ThetaScan.forward

    def forward(self, x):
        if self.cfg.backend != "b200":
            return original_forward(self, x)
        if not x.is_cuda:
            raise RuntimeError("b200 backend requires CUDA tensors")
        fused = _fused_core(self)
        if fused is None:
            return original_forward(self, x)
        return fused(x)

    block.ThetaScan.forward = forward
    _INSTALLED = True


def _fused_core(module):
    """A ThetaScanCore sharing ``module``'s parameters, or None if the core
    configuration is outside the fused path (the scan-level path then runs)."""
    cached = getattr(module, "_b200_fused", None)
    if cached is not None:
        # Parameters are shared objects and follow module.to(); buffers are
        # replaced by it, so hand the view the module's current ones.
        for name, buf in module.named_buffers():
            if name.startswith("_expand_"):
                cached._buffers[name] = buf
        return cached
    cfg = module.cfg
    if cfg.write_rule != "kernel" or not cfg.read_norm or cfg.read_norm_mode != "key_mass":
        return None
    if cfg.decay_gate != "off" or (cfg.read_fade and cfg.read_fade_mode != "fast") or cfg.value_centers:
        return None
    if cfg.rope != "none" and cfg.rope_placement != "input":
        return None
    from .config import KernelConfig, RoPEConfig, TemporalConfig, ThetaScanConfig
    from .mixer import ThetaScanCore
    kernel = KernelConfig(
        feature_map=cfg.kernel_kind, kernel_sharpness=float(cfg.softmax_gain),
        kernel_sharpness_mode=cfg.softmax_gain_mode, score_bias=bool(cfg.kernel_score_bias),
        relu2_threshold_mode=cfg.kernel_relu2_threshold_mode, bspline_basis_count=cfg.bspline_basis_count,
        bspline_bound=float(cfg.bspline_bound), bspline_scale=float(cfg.bspline_scale),
        bspline_scale_mode=cfg.bspline_scale_mode,
        value_representation="value_mlp" if cfg.value_mlp_mult > 0 else "raw",
        value_mlp_multiplier=float(cfg.value_mlp_mult) if cfg.value_mlp_mult > 0 else 1.0,
        sparsity=cfg.kernel_sparsity, sparse_blend_init=float(cfg.kernel_sparse_blend_init),
        relative_threshold_init=float(cfg.kernel_relative_threshold_init),
        threshold_temperature=float(cfg.kernel_threshold_temperature))
    temporal = TemporalConfig(mode="bank", recency_branches=cfg.fade_branches,
                              retention_inits=tuple(cfg.resolved_fade_alphas),
                              blend_mode=cfg.fade_blend_mode) if cfg.read_fade else TemporalConfig()
    public = ThetaScanConfig(
        d_model=cfg.d_model, n_heads=cfg.n_heads, head_dim=cfg.head_dim, memory_multiplier=cfg.mem_mult,
        feature_expansion=cfg.feature_expansion, expansion_key=cfg.expansion_key, depth=1,
        share_key_query=cfg.share_kq, key_value_heads=cfg.key_value_heads, output_gate=cfg.out_gate,
        family="kernel", kernel=kernel,
        rope=RoPEConfig(mode=cfg.rope, fraction=cfg.rope_frac, base=cfg.rope_base),
        temporal=temporal)
    if public.unsupported_reason() is not None:
        return None
    import torch
    with torch.random.fork_rng(devices=[]):
        # Construction draws initial weights; keep the caller's RNG stream intact.
        core = ThetaScanCore(public).to(next(module.parameters()).device)
    # Share storage: the fused view reads the reference module's parameters.
    for name, param in module.named_parameters():
        owner, _, leaf = name.rpartition(".")
        target = core.get_submodule(owner) if owner else core
        if hasattr(target, leaf):
            setattr(target, leaf, param)
    for name, buf in module.named_buffers():
        if name.startswith("_expand_"):
            core._buffers[name] = buf
    object.__setattr__(module, "_b200_fused", core)
    return core
