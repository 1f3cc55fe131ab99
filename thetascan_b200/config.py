"""Public configuration of the B200 ThetaScan mixer.

The field names, defaults and meaning follow the reference's public config
(src/thetascan/config.py:58-890: ``GNConfig``, ``KernelConfig``,
``RoPEConfig``, ``TemporalConfig``, ``RegularizationConfig``,
``RuntimeConfig``, ``ThetaScanConfig`` with ``to_dict`` / ``from_dict`` and
the versioned presets), so a manifest written for the reference loads here
unchanged.  ``RuntimeConfig.backend`` additionally accepts ``"b200"``; this
package executes that backend only (``"auto"`` resolves to it).

Validation restates the reference's rules for the fields this package reads
and raises ``NotImplementedError`` for configurations the GPU path does not
cover (EMA decay gates, value anchors, feature-space RoPE).
"""
from __future__ import annotations

import math
from copy import deepcopy
from dataclasses import asdict, dataclass, field
from numbers import Real
from typing import Any, Mapping

BACKENDS = ("auto", "naive", "quad", "chunk", "cumsum", "fla", "b200")


def _strict_int(name, value):
    if type(value) is not int:
        raise TypeError(f"{name} must be an integer")


def _strict_bool(name, value):
    if type(value) is not bool:
        raise TypeError(f"{name} must be a boolean")


def _finite(name, value):
    if isinstance(value, bool) or not isinstance(value, Real):
        raise TypeError(f"{name} must be a real number")
    if not math.isfinite(float(value)):
        raise ValueError(f"{name} must be finite")


@dataclass
class GNConfig:
    """Gauss--Newton fast-weight memory options (reference config.py:58-94)."""

    nonlinearity: str = "relu2"
    jacobian_steps: int = 1
    read_normalization: str = "none"
    # Extension beyond the reference (whose public config exposes neither):
    # "tanh" as a GN nonlinearity (h = tanh(pre), sigma' = 1 - h^2, the
    # pattern of the reference's nonlinearity table, nonlin.py:28-31; signed,
    # so only with read_normalization "none"), and `damping`, the GN family's
    # core epsilon (the reference's cfg.eps, _core/config.py:191: the damping
    # of the lambda solve, engine.py:255, and the epsilon of the q/k L2 norm,
    # the RMS norms and the read normalizations).  None keeps 1e-6.
    damping: float | None = None

    def validate(self) -> None:
        _strict_int("GNConfig.jacobian_steps", self.jacobian_steps)
        if self.nonlinearity not in ("relu2", "relu2_threshold", "silu", "swiglu", "tanh"):
            raise ValueError(f"unknown GN nonlinearity: {self.nonlinearity!r}")
        if self.damping is not None:
            _finite("GNConfig.damping", self.damping)
            if not self.damping > 0:
                raise ValueError("GNConfig.damping must be positive")
        if self.jacobian_steps not in (1, 2):
            raise ValueError("GNConfig.jacobian_steps must be 1 or 2")
        if self.read_normalization not in ("none", "w2_feature_mass", "both_feature_mass"):
            raise ValueError(f"unknown GN read normalization: {self.read_normalization!r}")
        if self.read_normalization != "none" and self.nonlinearity not in ("relu2", "relu2_threshold"):
            raise ValueError("GN feature-mass normalization requires relu2 or relu2_threshold")
        if self.read_normalization != "none" and self.jacobian_steps != 1:
            raise ValueError("GN feature-mass normalization requires jacobian_steps=1")


@dataclass
class KernelConfig:
    """Normalized positive-feature kernel memory (reference config.py:97-263)."""

    feature_map: str = "softmax_partition"
    value_representation: str = "raw"
    value_anchors: int = 8
    value_mlp_multiplier: float = 1.0
    kernel_sharpness: float = 8.0
    kernel_sharpness_mode: str = "fixed"
    score_bias: bool = False
    relu2_threshold_mode: str = "none"
    sparsity: str = "none"
    sparse_blend_init: float = 0.0
    relative_threshold_init: float = 0.01
    threshold_temperature: float = 0.25
    bspline_basis_count: int = 8
    bspline_degree: int = 3
    bspline_bound: float = 3.0
    bspline_scale: float = 1.0
    bspline_scale_mode: str = "fixed"
    feature_parameters_trainable: bool = True
    read_normalization: str = "key_mass"

    def validate(self) -> None:
        _strict_bool("KernelConfig.score_bias", self.score_bias)
        _strict_bool("KernelConfig.feature_parameters_trainable", self.feature_parameters_trainable)
        for name in ("value_anchors", "bspline_basis_count", "bspline_degree"):
            _strict_int(f"KernelConfig.{name}", getattr(self, name))
        for name in ("value_mlp_multiplier", "kernel_sharpness", "sparse_blend_init",
                     "relative_threshold_init", "threshold_temperature", "bspline_bound", "bspline_scale"):
            _finite(f"KernelConfig.{name}", getattr(self, name))
        if self.feature_map not in ("softmax_partition", "relu2_ridge", "projected_bspline"):
            raise ValueError(f"unknown kernel feature map: {self.feature_map!r}")
        if self.value_representation not in ("raw", "value_anchors", "value_mlp"):
            raise ValueError(f"unknown kernel value representation: {self.value_representation!r}")
        if self.read_normalization not in ("none", "key_mass", "feature_mass"):
            raise ValueError(f"unknown kernel read normalization: {self.read_normalization!r}")
        if self.kernel_sharpness <= 0:
            raise ValueError("KernelConfig.kernel_sharpness must be positive")
        if self.kernel_sharpness_mode not in ("fixed", "learned_per_head", "learned_per_feature"):
            raise ValueError("unknown KernelConfig.kernel_sharpness_mode")
        if self.sparsity not in ("none", "relative_soft", "relative_st", "relative_st_blend"):
            raise ValueError(f"unknown kernel sparsity: {self.sparsity!r}")
        if self.relu2_threshold_mode not in ("none", "learned_per_head"):
            raise ValueError("KernelConfig.relu2_threshold_mode must be 'none' or 'learned_per_head'")
        if self.relu2_threshold_mode != "none" and self.feature_map != "relu2_ridge":
            raise ValueError("learned relu2_threshold_mode requires feature_map='relu2_ridge'")
        if self.relu2_threshold_mode != "none" and self.score_bias:
            raise ValueError("relu2_threshold_mode and score_bias are redundant; enable only one")
        if self.sparsity != "none" and self.feature_map != "softmax_partition":
            raise ValueError("relative sparsity is defined for feature_map='softmax_partition' only")
        if self.kernel_sharpness_mode != "fixed" and self.feature_map != "softmax_partition":
            raise ValueError("learned kernel_sharpness_mode is defined for softmax_partition only")
        if self.bspline_basis_count <= self.bspline_degree:
            raise ValueError("kernel B-spline basis count must exceed its degree")
        if self.bspline_degree != 3:
            raise ValueError("kernel projected_bspline currently supports degree=3 only")
        if self.bspline_bound <= 0.0 or self.bspline_scale <= 0.0:
            raise ValueError("kernel B-spline bound and scale must be positive")
        if self.bspline_scale_mode not in ("fixed", "learned_per_head"):
            raise ValueError("KernelConfig.bspline_scale_mode must be 'fixed' or 'learned_per_head'")
        if self.feature_map != "projected_bspline" and self.bspline_scale_mode != "fixed":
            raise ValueError("learned bspline_scale_mode requires feature_map='projected_bspline'")


@dataclass
class RoPEConfig:
    """Rotary positions on memory keys/queries (reference config.py:266-294)."""

    mode: str = "none"
    fraction: float = 0.5
    base: float = 10_000.0
    placement: str = "input"

    def validate(self) -> None:
        _finite("RoPEConfig.fraction", self.fraction)
        _finite("RoPEConfig.base", self.base)
        if self.mode not in ("none", "partial", "full"):
            raise ValueError(f"unknown RoPE mode: {self.mode!r}")
        if self.placement not in ("input", "feature"):
            raise ValueError(f"unknown RoPE placement: {self.placement!r}")
        if not 0.0 < self.fraction <= 1.0:
            raise ValueError("RoPEConfig.fraction must be in (0, 1]")
        if self.base <= 0.0:
            raise ValueError("RoPEConfig.base must be positive")


@dataclass
class TemporalConfig:
    """Write combination over time (reference config.py:297-385)."""

    mode: str = "sum"
    bank_mode: str = "fast"
    retention_init: float = 0.9
    recency_branches: int = 1
    retention_inits: tuple[float, ...] | None = None
    half_life_inits: tuple[float, ...] | None = None
    blend_mode: str = "free"

    def resolved_retentions(self) -> tuple[float, ...]:
        """One retention per branch: explicit, from half-lives, or defaults."""
        if self.retention_inits is not None:
            return tuple(float(x) for x in self.retention_inits)
        if self.half_life_inits is not None:
            return tuple(math.pow(2.0, -1.0 / float(x)) for x in self.half_life_inits)
        if self.recency_branches == 2:
            return (float(self.retention_init), 0.99)
        return (float(self.retention_init),)

    def validate(self) -> None:
        _strict_int("TemporalConfig.recency_branches", self.recency_branches)
        _finite("TemporalConfig.retention_init", self.retention_init)
        if self.mode not in ("sum", "ema", "bank"):
            raise ValueError(f"unknown temporal mode: {self.mode!r}")
        if self.bank_mode not in ("fast", "stale"):
            raise ValueError(f"unknown bank mode: {self.bank_mode!r}")
        if not 0.0 < self.retention_init < 1.0:
            raise ValueError("TemporalConfig.retention_init must be in (0, 1)")
        # The reference accepts 1 or 2 branches; 3 (explicit initializers only)
        # is this package's extension for the four-view bank of config 4.
        if self.recency_branches not in (1, 2, 3):
            raise ValueError("TemporalConfig.recency_branches must be 1, 2 or 3")
        if self.blend_mode not in ("free", "tanh"):
            raise ValueError("TemporalConfig.blend_mode must be 'free' or 'tanh'")
        if self.retention_inits is not None and self.half_life_inits is not None:
            raise ValueError("set only one of retention_inits and half_life_inits")
        for name in ("retention_inits", "half_life_inits"):
            values = getattr(self, name)
            if values is not None:
                for i, x in enumerate(values):
                    _finite(f"TemporalConfig.{name}[{i}]", x)
        if self.half_life_inits is not None and any(x <= 0.0 for x in self.half_life_inits):
            raise ValueError("half-lives must be positive")
        retentions = self.resolved_retentions()
        if len(retentions) != self.recency_branches:
            raise ValueError("retention/half-life initializers must contain exactly recency_branches values")
        if any(not 0.0 < x < 1.0 for x in retentions):
            raise ValueError("retentions must be in (0, 1)")
        if self.recency_branches >= 2 and len(set(retentions)) != len(retentions):
            raise ValueError("recency branches require distinct initial timescales")


@dataclass
class RegularizationConfig:
    """Optional cosine-orthogonality penalties (reference config.py:388-406)."""

    feature_weight: float = 0.0
    head_weight: float = 0.0
    value_mlp_weight: float = 0.0

    def validate(self) -> None:
        for name in ("feature_weight", "head_weight", "value_mlp_weight"):
            _finite(f"RegularizationConfig.{name}", getattr(self, name))
            if getattr(self, name) < 0.0:
                raise ValueError("regularization weights must be non-negative")


@dataclass
class RuntimeConfig:
    """Execution selection (reference config.py:409-468) plus ``"b200"``."""

    backend: str = "auto"
    scan_chunk: int = 512

    def validate(self) -> None:
        if self.backend not in BACKENDS:
            raise ValueError("RuntimeConfig.backend must be one of " + ", ".join(repr(b) for b in BACKENDS))
        if isinstance(self.scan_chunk, bool) or not isinstance(self.scan_chunk, int):
            raise TypeError("RuntimeConfig.scan_chunk must be an int")
        if self.scan_chunk < 1:
            raise ValueError("RuntimeConfig.scan_chunk must be >= 1")


@dataclass
class ThetaScanConfig:
    """Public mixer configuration (reference config.py:471-796)."""

    d_model: int = 512
    n_heads: int = 8
    head_dim: int | None = None
    memory_multiplier: int = 2
    feature_expansion: int = 1
    expansion_key: str = "thetascan"
    depth: int = 1
    share_key_query: bool = False
    key_value_heads: int | None = None
    output_gate: bool = True
    family: str = "gn"
    gn: GNConfig = field(default_factory=GNConfig)
    kernel: KernelConfig = field(default_factory=KernelConfig)
    rope: RoPEConfig = field(default_factory=RoPEConfig)
    temporal: TemporalConfig = field(default_factory=TemporalConfig)
    regularization: RegularizationConfig = field(default_factory=RegularizationConfig)
    runtime: RuntimeConfig = field(default_factory=RuntimeConfig)

    @property
    def resolved_head_dim(self) -> int:
        return self.head_dim or self.d_model // self.n_heads

    @property
    def memory_width(self) -> int:
        """Effective feature width m = memory_multiplier * head_dim."""
        return self.memory_multiplier * self.resolved_head_dim

    def validate(self) -> None:
        _strict_bool("ThetaScanConfig.share_key_query", self.share_key_query)
        _strict_bool("ThetaScanConfig.output_gate", self.output_gate)
        for name in ("d_model", "n_heads", "memory_multiplier", "feature_expansion", "depth"):
            _strict_int(f"ThetaScanConfig.{name}", getattr(self, name))
        if self.head_dim is not None:
            _strict_int("ThetaScanConfig.head_dim", self.head_dim)
        if self.family not in ("gn", "kernel"):
            raise ValueError("ThetaScanConfig.family must be 'gn' or 'kernel'")
        if self.d_model <= 0 or self.n_heads <= 0 or self.memory_multiplier <= 0:
            raise ValueError("d_model, n_heads, and memory_multiplier must be positive")
        if self.d_model % self.n_heads:
            raise ValueError("d_model must be divisible by n_heads")
        if self.head_dim is not None and self.head_dim * self.n_heads != self.d_model:
            raise ValueError("head_dim * n_heads must equal d_model")
        if self.key_value_heads is not None:
            if type(self.key_value_heads) is not int:
                raise TypeError("ThetaScanConfig.key_value_heads must be an integer or None")
            if not 1 <= self.key_value_heads <= self.n_heads:
                raise ValueError("key_value_heads must be in [1, n_heads]")
            if self.n_heads % self.key_value_heads:
                raise ValueError("n_heads must be divisible by key_value_heads")
            if self.share_key_query:
                raise ValueError("key_value_heads and share_key_query=True are mutually exclusive")
        if self.depth < 1:
            raise ValueError("depth must be at least 1")
        if self.feature_expansion < 1:
            raise ValueError("ThetaScanConfig.feature_expansion must be >= 1")
        if self.feature_expansion > 1:
            if not isinstance(self.expansion_key, str) or not self.expansion_key:
                raise ValueError("ThetaScanConfig.expansion_key must be a non-empty string")
            if self.memory_width % self.feature_expansion:
                raise ValueError("feature_expansion must divide the effective memory width")
            if self.family == "gn" and self.gn.nonlinearity not in ("relu2", "relu2_threshold"):
                raise ValueError("GN feature_expansion requires nonlinearity 'relu2' or 'relu2_threshold'")
            if self.family == "kernel" and self.kernel.feature_map != "relu2_ridge":
                raise ValueError("kernel feature_expansion requires feature_map='relu2_ridge'")
        self.temporal.validate()
        self.rope.validate()
        self.regularization.validate()
        self.runtime.validate()
        if self.runtime.backend == "cumsum" and self.temporal.mode != "sum":
            raise ValueError("backend='cumsum' supports temporal.mode='sum' only")
        if self.family == "gn":
            self.gn.validate()
            if self.rope.mode != "none" and self.rope.placement == "feature" and \
                    self.gn.read_normalization != "none":
                raise ValueError("feature-space RoPE makes the GN feature-mass denominator signed")
        else:
            k = self.kernel
            k.validate()
            if self.rope.mode != "none" and self.rope.placement == "feature" and \
                    k.read_normalization in ("key_mass", "feature_mass"):
                raise ValueError("feature-space RoPE makes the kernel normalization denominator signed")
            if self.depth != 1:
                raise ValueError("kernel memory currently supports depth=1 only")
            if k.feature_map == "projected_bspline":
                if self.memory_width % k.bspline_basis_count:
                    raise ValueError("projected_bspline requires memory_multiplier * head_dim "
                                     "to be divisible by bspline_basis_count")
                if k.score_bias:
                    raise ValueError("score_bias is not used by projected_bspline")
            if k.value_representation == "value_anchors" and k.read_normalization != "key_mass":
                raise ValueError("kernel value_anchors requires read_normalization='key_mass'")

    def to_dict(self) -> dict[str, Any]:
        """Detached manifest (reference config.py:633-640)."""
        return deepcopy(asdict(self))

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> "ThetaScanConfig":
        """Build from a nested manifest, optionally starting from a preset
        (reference config.py:642-701)."""
        if not isinstance(data, Mapping):
            raise TypeError("ThetaScanConfig.from_dict expects a mapping")
        payload: dict[str, Any] = deepcopy(dict(data))

        def merge(base, over):
            for key, value in over.items():
                if isinstance(value, Mapping) and isinstance(base.get(key), dict):
                    base[key] = merge(dict(base[key]), value)
                else:
                    base[key] = deepcopy(value)
            return base

        preset = payload.pop("preset", None)
        if preset is not None:
            presets = {"gn_reference_v0_1": cls.gn_reference_v0_1,
                       "gn_expanded_reference_v0_1": cls.gn_expanded_reference_v0_1,
                       "kernel_expanded_reference_v0_1": cls.kernel_expanded_reference_v0_1}
            if preset not in presets:
                raise ValueError(f"unknown ThetaScan preset: {preset!r}")
            d_model = payload.pop("d_model", 512)
            n_heads = payload.pop("n_heads", 8)
            payload = merge(presets[preset](d_model=d_model, n_heads=n_heads).to_dict(), payload)
        nested = {"gn": GNConfig, "kernel": KernelConfig, "rope": RoPEConfig, "temporal": TemporalConfig,
                  "regularization": RegularizationConfig, "runtime": RuntimeConfig}
        for name, ctor in nested.items():
            value = payload.get(name)
            if isinstance(value, Mapping):
                item = dict(value)
                if name == "temporal":
                    for key in ("retention_inits", "half_life_inits"):
                        if item.get(key) is not None:
                            item[key] = tuple(item[key])
                payload[name] = ctor(**item)
        config = cls(**payload)
        config.validate()
        return config

    # Versioned presets (reference config.py:804-890).
    @classmethod
    def gn_reference_v0_1(cls, d_model: int = 512, n_heads: int = 8) -> "ThetaScanConfig":
        return cls(d_model=d_model, n_heads=n_heads, memory_multiplier=3, share_key_query=True,
                   output_gate=False, family="gn",
                   gn=GNConfig(nonlinearity="relu2", jacobian_steps=1, read_normalization="both_feature_mass"),
                   rope=RoPEConfig(mode="partial", fraction=0.5, base=10_000.0),
                   temporal=TemporalConfig(mode="bank", bank_mode="fast", retention_init=0.9, recency_branches=1,
                                           retention_inits=(0.9,), blend_mode="free"))

    @classmethod
    def gn_expanded_reference_v0_1(cls, d_model: int = 512, n_heads: int = 8) -> "ThetaScanConfig":
        return cls(d_model=d_model, n_heads=n_heads, memory_multiplier=6, feature_expansion=2,
                   share_key_query=True, output_gate=False, family="gn",
                   gn=GNConfig(nonlinearity="relu2_threshold", jacobian_steps=1,
                               read_normalization="both_feature_mass"),
                   rope=RoPEConfig(mode="partial", fraction=0.5, base=10_000.0),
                   temporal=TemporalConfig(mode="bank", bank_mode="fast", recency_branches=1,
                                           retention_inits=(0.9,), blend_mode="free"))

    @classmethod
    def kernel_expanded_reference_v0_1(cls, d_model: int = 512, n_heads: int = 8) -> "ThetaScanConfig":
        return cls(d_model=d_model, n_heads=n_heads, memory_multiplier=6, feature_expansion=2,
                   share_key_query=True, output_gate=False, family="kernel",
                   kernel=KernelConfig(feature_map="relu2_ridge", relu2_threshold_mode="learned_per_head",
                                       read_normalization="key_mass"),
                   rope=RoPEConfig(mode="partial", fraction=0.5, base=10_000.0),
                   temporal=TemporalConfig(mode="bank", bank_mode="fast", recency_branches=2,
                                           half_life_inits=(8.0, 64.0), blend_mode="free"))

    def unsupported_reason(self) -> str | None:
        """Why the B200 path cannot run this (validated) config, or None."""
        if self.runtime.backend not in ("auto", "b200"):
            return f"this package executes backend 'b200' only, not {self.runtime.backend!r}"
        if self.temporal.mode == "ema":
            return "the data-dependent EMA decay gate is not built"
        if self.rope.mode != "none" and self.rope.placement == "feature":
            return "feature-space RoPE is not built"
        if self.family == "gn":
            return None
        k = self.kernel
        if k.value_representation == "value_anchors":
            return "kernel value_anchors are not built"
        return None
