"""Oracle for the per-token nonlinear pieces of the write/read.

RMSNorm / L2 norm (reference ``_core/modules/norms.py:5-12``), RoPE
(``_core/modules/rope.py:7-72``) and the three positive kernel feature maps of
``_core/ops/kernel_features.py``.  Test infrastructure only.
"""
from __future__ import annotations

import math

import torch


def rmsnorm(a, eps: float = 1e-6):
    """``(a * inv, inv)`` with ``inv = rsqrt(mean(a^2) + eps)`` (norms.py:5-8)."""
    inv = torch.rsqrt(a.pow(2).mean(-1, keepdim=True) + eps)
    return a * inv, inv


def l2norm(x, eps: float = 1e-6):
    """``x / max(||x||, eps)`` (norms.py:11-12)."""
    return x / x.norm(dim=-1, keepdim=True).clamp_min(eps)


def rope_rotation_width(d: int, mode: str, frac: float) -> int:
    """Rotated channel count (rope.py:61-65): all pairs, or ``frac`` of them."""
    if mode == "none":
        return 0
    max_rot = d // 2 * 2
    if max_rot == 0:
        return 0
    if mode == "full":
        return max_rot
    return min(max_rot, max(2, int(d * frac) // 2 * 2))


def rope_tables(T: int, rot: int, base: float, dtype=torch.float64):
    """``cos/sin [T, rot/2]`` with phases in at least float32 (rope.py:7-38)."""
    phase = torch.float64 if dtype == torch.float64 else torch.float32
    inv = 1.0 / (base ** (torch.arange(0, rot, 2, dtype=phase) / rot))
    angles = torch.outer(torch.arange(T, dtype=phase), inv)
    return angles.cos().to(dtype), angles.sin().to(dtype)


def apply_rope(x, mode: str, frac: float, base: float):
    """Rotate the first ``rot`` channels of ``x [B,H,T,d]`` in adjacent pairs.

    Pair ``(x[2p], x[2p+1])`` turns by ``t * base^(-2p/rot)`` (rope.py:57-72).
    """
    rot = rope_rotation_width(x.shape[-1], mode, frac)
    if rot == 0:
        return x
    cos, sin = rope_tables(x.shape[2], rot, base, x.dtype)
    even, odd = x[..., 0:rot:2], x[..., 1:rot:2]
    rotated = torch.stack((even * cos - odd * sin, even * sin + odd * cos), dim=-1)
    return torch.cat((rotated.flatten(-2), x[..., rot:]), dim=-1)


def _per_head(value, ref):
    """Broadcast a ``[H]`` or ``[H,M]`` control (kernel_features.py:12-31)."""
    value = value.to(ref.dtype)
    if value.ndim == 1:
        return value.view(1, -1, *([1] * (ref.ndim - 2)))
    return value.view(1, value.shape[0], *([1] * (ref.ndim - 3)), value.shape[1])


def relu2_ridge(pre, *, score_bias=None, threshold=None, eps: float = 1e-6):
    """``relu(pre + b - tau)^2 / sum``, uniform row if the sum is ``<= eps``.

    Restates ``relu2_ridge_features`` (kernel_features.py:116-135).
    """
    if score_bias is not None:
        pre = pre + _per_head(score_bias, pre)
    if threshold is not None:
        pre = pre - _per_head(threshold, pre)
    feats = torch.relu(pre).square()
    mass = feats.sum(-1, keepdim=True)
    uniform = torch.full_like(feats, 1.0 / feats.shape[-1])
    return torch.where(mass > eps, feats / mass.clamp_min(eps), uniform)


def relative_threshold(logits, rho, *, temperature: float, straight_through: bool, eps: float):
    """Relative-to-max sparse simplex (kernel_features.py:43-70)."""
    shifted = logits - logits.amax(-1, keepdim=True)
    margin = shifted - _per_head(rho, logits).clamp(min=eps, max=1.0 - eps).log()
    soft = torch.sigmoid(margin / temperature)
    gate = soft
    if straight_through:
        gate = (margin >= 0.0).to(soft.dtype) + soft - soft.detach()
    weights = shifted.exp() * gate
    return weights / weights.sum(-1, keepdim=True).clamp_min(eps)


def softmax_partition(pre, *, gain=8.0, score_bias=None, sparsity: str = "none",
                      rho=None, blend=None, temperature: float = 0.25, eps: float = 1e-6):
    """``softmax(gain * (pre + b))`` with optional relative sparsity.

    Restates ``softmax_partition_features`` (kernel_features.py:73-113).
    ``gain`` is a float or a ``[H]`` / ``[H,M]`` tensor.
    """
    scores = pre if score_bias is None else pre + _per_head(score_bias, pre)
    g = gain if not torch.is_tensor(gain) else _per_head(gain, scores)
    logits = scores * g
    dense = torch.softmax(logits, -1)
    if sparsity == "none":
        return dense
    sparse = relative_threshold(
        logits, rho, temperature=temperature,
        straight_through=sparsity in ("relative_st", "relative_st_blend"), eps=eps,
    )
    if sparsity != "relative_st_blend":
        return sparse
    return dense + _per_head(blend, logits) * (sparse - dense)


def open_uniform_knots(n_basis: int, degree: int, bound: float, dtype=torch.float64):
    """Clamped knot vector: ``degree+1`` copies of each end and ``n-d-1``
    uniform interior knots (kernel_features.py:162-172)."""
    inner = n_basis - degree - 1
    interior = torch.linspace(-bound, bound, inner + 2, dtype=dtype)[1:-1] if inner else torch.empty(0, dtype=dtype)
    ends = torch.full((degree + 1,), bound, dtype=dtype)
    return torch.cat([-ends, interior, ends])


def bspline_basis(coords, *, n_basis: int, degree: int = 3, bound: float = 3.0):
    """Open-uniform B-spline basis by the Cox--de Boor recursion.

    Restates ``open_uniform_bspline_basis`` (kernel_features.py:138-205):
    clamp to ``[-bound, nextafter(bound, -bound)]``, half-open degree-0 spans,
    zero-denominator terms dropped, then clamp negatives and renormalise.
    """
    dtype = coords.dtype
    knots = open_uniform_knots(n_basis, degree, bound, dtype)
    high = torch.tensor(bound, dtype=dtype)
    x = torch.minimum(coords.clamp(-bound, bound), torch.nextafter(high, -high))
    xe = x.unsqueeze(-1)
    basis = ((xe >= knots[:-1]) & (xe < knots[1:])).to(dtype)
    tiny = torch.finfo(dtype).tiny
    for order in range(1, degree + 1):
        count = knots.numel() - order - 1
        left_den = knots[order:order + count] - knots[:count]
        right_den = knots[order + 1:order + 1 + count] - knots[1:1 + count]
        left = torch.where(left_den > 0, (xe - knots[:count]) / left_den.clamp_min(tiny),
                           torch.zeros_like(left_den))
        right = torch.where(right_den > 0,
                            (knots[order + 1:order + 1 + count] - xe) / right_den.clamp_min(tiny),
                            torch.zeros_like(right_den))
        basis = left * basis[..., :count] + right * basis[..., 1:count + 1]
    basis = basis.clamp_min(0.0)
    return basis / basis.sum(-1, keepdim=True).clamp_min(tiny)


def projected_bspline(pre, *, n_basis: int, degree: int = 3, bound: float = 3.0, scale=1.0):
    """Per-projection B-spline partition, concatenated and divided by P.

    Restates ``projected_bspline_features`` (kernel_features.py:208-230).
    """
    s = scale if not torch.is_tensor(scale) else _per_head(scale, pre)
    basis = bspline_basis(pre * s, n_basis=n_basis, degree=degree, bound=bound)
    return basis.flatten(-2) / float(pre.shape[-1])


def feature_map(pre, spec: dict):
    """Dispatch on ``spec['kind']`` (kernel_features.py:233-273)."""
    kind = spec["kind"]
    eps = spec.get("eps", 1e-6)
    if kind == "relu2_ridge":
        return relu2_ridge(pre, score_bias=spec.get("score_bias"),
                           threshold=spec.get("relu2_threshold"), eps=eps)
    if kind == "softmax_partition":
        return softmax_partition(
            pre, gain=spec.get("gain", 8.0), score_bias=spec.get("score_bias"),
            sparsity=spec.get("sparsity", "none"), rho=spec.get("rho"),
            blend=spec.get("blend"), temperature=spec.get("temperature", 0.25), eps=eps,
        )
    if kind == "projected_bspline":
        return projected_bspline(pre, n_basis=spec["n_basis"], degree=spec.get("degree", 3),
                                 bound=spec.get("bound", 3.0), scale=spec.get("scale", 1.0))
    raise ValueError(f"unknown kernel kind: {kind!r}")


def inverse_softplus(value: float) -> float:
    """Scalar inverse of softplus (block.py:24-26)."""
    return value + math.log(-math.expm1(-value))
