"""Float32 kernel-family hot path (the reference's fp32 configuration).

The reference runs its fp32 configuration (softmax-partition features,
B=2, T=512, d_model=256, H=4) in float32 end to end, and the parity bound
there is rel-err 1e-5: out of reach of bf16 (2^-9) or tf32 (2^-11)
tensor-core operands.  For a float32 input the mixer therefore runs

* every read over the sequence -- the key-mass scans [phi(q).S | phi(q).z],
  the per-feature mass prefix sums, the unnormalized reads -- on the float32
  scan kernels (``ts_b200_scan_fwd/bwd`` with ``f32_streams``: f32 FMAs on
  the CUDA cores), through :func:`thetascan_b200.scan.linattn_views`;
* the per-token math around them -- rmsnorm(W1 x), the feature map, the slow
  decode W2 phi(q), the read division and the view blend -- in float32
  PyTorch on the same device, under autograd.

Float32 GEMMs follow PyTorch's matmul precision setting; its default (IEEE
float32, TF32 off) is what the 1e-5 bound needs.  This restates the kernel
write rule of the reference: engine.py:117-158 (features), 260-553 (write,
dual read, key-mass / feature-mass / unnormalized reads) and block.py:644-718
(the temporal bank blend), with the feature maps of kernel_features.py:
73-273.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from .scan import linattn_views
from .seqpar import sharded_reads


def _rmsnorm(a: torch.Tensor, eps: float) -> torch.Tensor:
    """``a * rsqrt(mean(a^2) + eps)`` (norms.py:5-8)."""
    return a * torch.rsqrt(a.square().mean(-1, keepdim=True) + eps)


def _head_control(value: torch.Tensor, ref: torch.Tensor) -> torch.Tensor:
    """A ``[H]`` or ``[H, m]`` control broadcast against ``[B,H,T,...]``
    (kernel_features.py:12-31)."""
    if value.ndim == 1:
        return value.view(1, -1, *([1] * (ref.ndim - 2)))
    return value.view(1, value.shape[0], *([1] * (ref.ndim - 3)), value.shape[1])


def _bspline_partition(coords: torch.Tensor, n_basis: int, bound: float, degree: int = 3) -> torch.Tensor:
    """Open-uniform cubic B-spline basis by the Cox--de Boor recursion, clamped
    into ``[-bound, bound)``, negatives clamped and rows renormalised
    (kernel_features.py:138-205)."""
    dt = coords.dtype
    inner = n_basis - degree - 1
    interior = torch.linspace(-bound, bound, inner + 2, dtype=dt, device=coords.device)[1:-1]
    ends = torch.full((degree + 1,), bound, dtype=dt, device=coords.device)
    knots = torch.cat([-ends, interior, ends])
    top = torch.tensor(bound, dtype=dt, device=coords.device)
    x = torch.minimum(coords.clamp(-bound, bound), torch.nextafter(top, -top)).unsqueeze(-1)
    basis = ((x >= knots[:-1]) & (x < knots[1:])).to(dt)
    tiny = torch.finfo(dt).tiny
    for order in range(1, degree + 1):
        n = knots.numel() - order - 1
        lo, hi = knots[:n], knots[order + 1:order + 1 + n]
        lden, rden = knots[order:order + n] - lo, hi - knots[1:1 + n]
        left = torch.where(lden > 0, (x - lo) / lden.clamp_min(tiny), torch.zeros_like(lden))
        right = torch.where(rden > 0, (hi - x) / rden.clamp_min(tiny), torch.zeros_like(rden))
        basis = left * basis[..., :n] + right * basis[..., 1:n + 1]
    basis = basis.clamp_min(0.0)
    return basis / basis.sum(-1, keepdim=True).clamp_min(tiny)


def features(x, W1, spec, ctl) -> torch.Tensor:
    """``phi(rmsnorm(W1 x))`` for ``x [B,H,T,d]`` and ``W1 [H,P,d]``."""
    pre = _rmsnorm(torch.einsum("hpd,bhtd->bhtp", W1, x), spec.eps)
    if spec.kind == "relu2_ridge":
        if ctl.get("score_bias") is not None:
            pre = pre + _head_control(ctl["score_bias"], pre)
        if ctl.get("threshold") is not None:
            pre = pre - _head_control(ctl["threshold"], pre)
        feats = torch.relu(pre).square()
        mass = feats.sum(-1, keepdim=True)
        return torch.where(mass > spec.eps, feats / mass.clamp_min(spec.eps),
                           torch.full_like(feats, 1.0 / feats.shape[-1]))
    if spec.kind == "softmax_partition":
        if ctl.get("score_bias") is not None:
            pre = pre + _head_control(ctl["score_bias"], pre)
        gain = ctl.get("gain")
        logits = pre * (spec.gain if gain is None else _head_control(gain, pre))
        dense = torch.softmax(logits, -1)
        if spec.sparsity == "none":
            return dense
        # relative sparsity (kernel_features.py:43-70, 95-113)
        shifted = logits - logits.amax(dim=-1, keepdim=True)
        rho = _head_control(ctl["relative_threshold"], logits).clamp(min=spec.eps, max=1.0 - spec.eps)
        margin = shifted - rho.log()
        soft = torch.sigmoid(margin / spec.temperature)
        if spec.sparsity == "relative_soft":
            gate = soft
        else:
            gate = (margin >= 0.0).to(soft.dtype) + soft - soft.detach()
        weights = shifted.exp() * gate
        sparse = weights / weights.sum(-1, keepdim=True).clamp_min(spec.eps)
        if spec.sparsity != "relative_st_blend":
            return sparse
        return dense + _head_control(ctl["sparse_blend"], logits) * (sparse - dense)
    if spec.kind == "projected_bspline":
        scale = ctl.get("spline_scale")
        s = spec.spline_scale if scale is None else _head_control(scale, pre)
        basis = _bspline_partition(pre * s, spec.basis, spec.bound)
        return basis.flatten(-2) / float(pre.shape[-1])
    raise NotImplementedError(f"b200 float32 path: feature map {spec.kind!r}")


def _views_fn(shard):
    """The multi-view scan of this call: the float32 kernels over the whole
    sequence, or, on a sequence shard, the shard's reads entering with the
    earlier shards' state (payloads cut to the kernels' 256 columns with the
    exchange's unit column)."""
    if shard is None:
        return linattn_views

    def views(query, keys, payload, rets, append_unit=False, stale=None):
        width = payload.shape[-1]
        step = 128 if width + 1 > 256 else width
        parts = []
        for start in range(0, width, step):
            unit = append_unit and start + step >= width
            piece = payload[..., start:start + step].contiguous()
            parts.append(sharded_reads(shard, linattn_views, query, keys, piece, rets, append_unit=unit,
                                       stale=stale))
        return [p[0] if len(p) == 1 else torch.cat(p, dim=-1) for p in zip(*parts)]

    return views


def _mass(phi_k, retention, stale, views=linattn_views):
    """Per-feature key mass of one view, ``sum_{j<=t} w(t-j) phi_k[j]``
    (view.mass_cum, interface.py:216-230, 278-279, 306-307), as a scan of
    ``phi_k`` with unit queries and keys."""
    one = phi_k.new_ones(*phi_k.shape[:3], 1)
    return views(one, one, phi_k, (retention,), stale=(stale,))[0]


def kernel_core_f32(q, k, v, W1, W2, spec, *, threshold=None, score_bias=None, gain=None, spline_scale=None,
                    log_alphas=None, etas=None, relative_threshold=None, sparse_blend=None, shard=None):
    """``y = q + W2 phi(q) + blended normalized memory``, float32, ``[B,H,T,d]``.

    Same arguments as :func:`thetascan_b200.kernel.kernel_core` with float32
    streams; ``log_alphas``/``etas`` are ``[J,H]`` for a bank.  ``shard`` (a
    :class:`thetascan_b200.seqpar.SeqShard`) makes the streams one contiguous
    slice of longer sequences: every view and read normalisation, each scan
    entering with the earlier slices' state."""
    for x in (q, k, v):
        if not x.is_cuda:
            raise RuntimeError("b200 backend requires CUDA tensors")
        if x.dtype != torch.float32:
            raise NotImplementedError("b200 float32 path: float32 streams only")
    if (log_alphas is None) != (spec.mode == "sum"):
        raise ValueError("kernel_core: log_alphas are required exactly for a bank (mode fast/stale)")
    ctl = {"threshold": threshold, "score_bias": score_bias, "gain": gain, "spline_scale": spline_scale,
           "relative_threshold": relative_threshold, "sparse_blend": sparse_blend}
    eps = spec.eps
    phi_k = features(k, W1, spec, ctl)
    phi_q = features(q, W1, spec, ctl)
    base = q + torch.einsum("hdm,bhtm->bhtd", W2, phi_q)
    J = 0 if log_alphas is None else log_alphas.shape[0]
    rets = (None,) + tuple(log_alphas[j] for j in range(J))
    stale = (False,) + (spec.mode == "stale",) * J
    views = _views_fn(shard)
    if spec.read == "key_mass":
        reads = views(phi_q, phi_k, v, rets, append_unit=True, stale=stale)
        mems = [r[..., :-1] / (r[..., -1:] + eps) for r in reads]
    elif spec.read == "feature_mass":
        mems = []
        for ret, st in zip(rets, stale):
            query = phi_q / (_mass(phi_k, ret, st, views) + eps)
            mems.append(views(query, phi_k, v, (ret,), stale=(st,))[0])
    elif spec.read == "none":
        mems = list(views(phi_q, phi_k, v, rets, stale=stale))
    else:
        raise ValueError(f"kernel_core: unknown read normalization {spec.read!r}")
    outs = [base + mem for mem in mems]
    y = outs[0]
    for j in range(J):
        eta = etas[j].view(1, -1, 1, 1)
        y = y + eta * (outs[1 + j] - outs[0]) if spec.mode == "fast" else y - eta * (outs[1 + j] - base)
    return y
