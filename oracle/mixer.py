"""Oracle for the kernel-family ThetaScan mixer: write, scan, normalized read.

The hot path (reference ``_core/ops/engine.py:260-553`` with the temporal
orchestration of ``_core/modules/block.py:644-718``) is restated by
:func:`kernel_core`; :func:`mixer_forward` wraps it with the projections,
RoPE, L2 norm, output gate and output projection of ``block.py:573-724``.
Test infrastructure only.
"""
from __future__ import annotations

import hashlib
import math

import torch
import torch.nn.functional as F

from . import features, scan


# --------------------------------------------------------------------------- views

def view_terms(mode: str, n_branches: int):
    """Scan terms of each temporal view as ``(coefficient, retention_slot)``.

    Slot 0 is the plain sum, slot ``1+j`` the static retention of branch ``j``.
    ``sum`` reads the plain view only; a ``fast`` bank adds one recency view per
    branch (``FadeFast.scan_terms``, interface.py:300-301); a ``stale`` bank adds
    ``sum - fast_j`` (``FadeStale.scan_terms``, interface.py:268-273).
    """
    views = [((1.0, 0),)]
    for j in range(n_branches):
        if mode == "fast":
            views.append(((1.0, 1 + j),))
        else:
            views.append(((1.0, 0), (-1.0, 1 + j)))
    return views


def blend_outputs(outs, base_out, mode: str, etas):
    """Combine per-view reads into the mixer read (block.py:676-718).

    ``fast``: ``y = out + sum_j eta_j (out_fast_j - out)``.
    ``stale``: ``y = out - sum_j eta_j (out_stale_j - out_base)``, where
    ``out_base`` is the zero-memory read.  ``etas`` is ``[J, H]``.
    """
    result = outs[0]
    for j in range(len(outs) - 1):
        eta = etas[j].view(1, -1, 1, 1).to(result.dtype)
        if mode == "fast":
            result = result + eta * (outs[1 + j] - outs[0])
        else:
            result = result - eta * (outs[1 + j] - base_out)
    return result


# --------------------------------------------------------------------------- core

def featurize(x, W1, spec, eps):
    """``phi(rmsnorm(W1 x))`` for ``x [B,H,T,d]``, ``W1 [H,P,d]``
    (engine.py:117-158 with ``act_norm`` on, kernel write rule)."""
    a = torch.einsum("hpd,bhtd->bhtp", W1, x)
    pre, _ = features.rmsnorm(a, eps)
    return features.feature_map(pre, dict(spec, eps=eps))


def kernel_core(q, k, v, W1, W2, spec, *, log_alphas=None, etas=None, mode="fast",
                read_norm="key_mass", eps=1e-6, chunk=512, scan_fn=None):
    """Kernel-family hot path: ``y = q + W2 phi(q) + blended normalized memory``.

    ``q, k, v`` are ``[B,H,T,d]`` after RoPE/L2 norm; ``W1 [H,P,d]`` and
    ``W2 [H,d,m]`` are the effective (expanded) weights; ``log_alphas`` and
    ``etas`` are ``[J,H]`` (``None`` for the plain sum view alone).

    Write: ``phi_k`` keys, raw ``v`` payload (engine.py:276-322).  Read: the
    shared query features and slow decode ``W2 phi_q`` (engine.py:522-528), then
    per view the key-mass normalized read ``corr[:d] / (corr[d] + eps)`` of the
    augmented payload ``[v | 1]`` (engine.py:419-442), the per-feature mass
    read (engine.py:443-456), or the unnormalized read (engine.py:402-416).
    ``scan_fn(q, k, v, retentions)`` defaults to the chunked oracle.
    """
    if scan_fn is None:
        scan_fn = lambda qq, kk, vv, rets: scan.linattn_chunk_views(qq, kk, vv, rets, chunk)
    phi_k = featurize(k, W1, spec, eps).to(v.dtype)
    phi_q = featurize(q, W1, spec, eps)
    base = torch.einsum("hdm,bhtm->bhtd", W2, phi_q)
    J = 0 if log_alphas is None else log_alphas.shape[0]
    retentions = [None] + [log_alphas[j] for j in range(J)]
    terms = view_terms(mode, J)

    def combine(scanned, view):
        total = None
        for coef, slot in view:
            piece = scanned[slot] if coef == 1.0 else coef * scanned[slot]
            total = piece if total is None else total + piece
        return total

    if read_norm == "key_mass":
        unit = torch.cat([v, v.new_ones(*v.shape[:3], 1)], dim=-1)
        scanned = scan_fn(phi_q.to(phi_k.dtype), phi_k, unit, tuple(retentions))
        mems = []
        for view in terms:
            corr = combine(scanned, view)
            mems.append(corr[..., :-1] / (corr[..., -1:] + eps))
    elif read_norm == "feature_mass":
        mems = []
        for view in terms:
            mass = None
            for coef, slot in view:
                r = retentions[slot]
                part = scan.causal_prefix_sum(phi_k) if r is None else scan.ema_cumsum(phi_k, r, chunk)
                part = part if coef == 1.0 else coef * part
                mass = part if mass is None else mass + part
            query = (phi_q / (mass + eps)).to(phi_k.dtype)
            scanned = scan_fn(query, phi_k, v, tuple(retentions))
            mems.append(combine(scanned, view))
    else:
        scanned = scan_fn(phi_q.to(phi_k.dtype), phi_k, v, tuple(retentions))
        mems = [combine(scanned, view) for view in terms]
    outs = [q + (base + mem) for mem in mems]
    return blend_outputs(outs, q + base, mode, etas) if J else outs[0]


# --------------------------------------------------------------------------- expansion maps

EXPANSION_DOMAIN = "thetascan-expansion-v1"


def rademacher(shape, *, key: str, role: str):
    """Key-derived +-1 signs: low bit of SHAKE-256 over a versioned domain
    string ``domain \\0 key \\0 role \\0 shape`` (block.py:49-74)."""
    count = math.prod(shape)
    domain = f"{EXPANSION_DOMAIN}\0{key}\0{role}\0{','.join(str(s) for s in shape)}".encode()
    raw = hashlib.shake_256(domain).digest(count)
    bits = torch.tensor(list(raw), dtype=torch.uint8)
    return (bits & 1).to(torch.float32).mul(2.0).sub(1.0).reshape(shape)


def row_map(shape, *, key: str, role: str):
    """Uncentred unit-norm rows of a sign map (block.py:117-133, center_rows=False)."""
    matrix = rademacher(shape, key=key, role=role)
    norm = matrix.norm(dim=-1, keepdim=True)
    fallback = rademacher(shape, key=key, role=f"{role}-fallback")
    matrix = torch.where(norm > 0.0, matrix, fallback)
    return matrix / matrix.norm(dim=-1, keepdim=True)


# --------------------------------------------------------------------------- full mixer

def effective_weights(p, cfg):
    """``W1_eff = U W1`` and ``W2_eff = W2 D`` (block.py:546-567, fp32 params)."""
    W1, W2 = p["W1.0"], p["W2.0"]
    if cfg.get("feature_expansion", 1) > 1:
        W1 = torch.matmul(p["_expand_w1_0"].to(W1.dtype), W1)
        W2 = torch.matmul(W2, p["_expand_w2_0"].to(W2.dtype))
    return W1, W2


def layer_weights(p, cfg):
    """Effective ``(W1, W2, Wg)`` of every block of a GN net (block.py:546-567)."""
    out = []
    for l in range(cfg.get("depth", 1)):
        W1, W2 = p[f"W1.{l}"], p[f"W2.{l}"]
        if cfg.get("feature_expansion", 1) > 1:
            W1 = torch.matmul(p[f"_expand_w1_{l}"].to(W1.dtype), W1)
            W2 = torch.matmul(W2, p[f"_expand_w2_{l}"].to(W2.dtype))
        out.append((W1, W2, p.get(f"Wg.{l}")))
    return out


def feature_spec(p, cfg):
    """Kernel controls of block.py:408-456 as an oracle ``spec`` dict."""
    kind = cfg["kernel_kind"]
    spec = {"kind": kind}
    if kind == "relu2_ridge":
        spec["relu2_threshold"] = p.get("kernel_relu2_threshold")
        spec["score_bias"] = p.get("kernel_score_bias")
    elif kind == "softmax_partition":
        raw = p.get("kernel_sharpness_raw")
        spec["gain"] = cfg.get("softmax_gain", 8.0) if raw is None else F.softplus(raw).clamp_min(
            torch.finfo(raw.dtype).tiny)
        spec["score_bias"] = p.get("kernel_score_bias")
        # relative sparsity (block.py:167-180, 421-438): rho = sigmoid(raw);
        # the blend's forward value clamp(raw, 0, 1), its gradient sigmoid's
        spec["sparsity"] = cfg.get("kernel_sparsity", "none")
        spec["temperature"] = cfg.get("kernel_threshold_temperature", 0.25)
        if p.get("kernel_relative_threshold_raw") is not None:
            spec["rho"] = torch.sigmoid(p["kernel_relative_threshold_raw"])
        raw_b = p.get("kernel_sparse_blend_raw")
        if raw_b is not None:
            sur = torch.sigmoid(raw_b)
            spec["blend"] = raw_b.clamp(0.0, 1.0).detach() + sur - sur.detach()
    else:
        raw = p.get("bspline_scale_raw")
        spec["n_basis"] = cfg["bspline_basis_count"]
        spec["bound"] = cfg.get("bspline_bound", 3.0)
        spec["scale"] = cfg.get("bspline_scale", 1.0) if raw is None else F.softplus(raw).clamp_min(
            torch.finfo(raw.dtype).tiny)
    return spec


def fade_parameters(p, cfg, dtype):
    """``log_alpha = -softplus(-raw)`` and ``eta`` (free or tanh) per branch,
    shaped ``[J, H]`` (block.py:483-494, 647-657)."""
    if not cfg.get("read_fade", False):
        return None, None
    raw, eta = p["fade_alpha"], p["fade_eta"]
    if raw.ndim == 1:
        raw, eta = raw.unsqueeze(0), eta.unsqueeze(0)
    if cfg.get("fade_blend_mode", "free") == "tanh":
        eta = torch.tanh(eta)
    return (-F.softplus(-raw)).to(dtype), eta


def project_qkv(p, cfg, x):
    """q, k, v ``[B,H,T,d]`` for the three projection layouts (block.py:577-594)."""
    B, T, _ = x.shape
    H, d = cfg["n_heads"], cfg["head_dim"]
    if cfg.get("key_value_heads") is not None:
        G = cfg["key_value_heads"]
        q = F.linear(x, p["proj_q.weight"]).view(B, T, H, d).transpose(1, 2)
        k = F.linear(x, p["proj_k.weight"]).view(B, T, G, d).transpose(1, 2)
        v = F.linear(x, p["proj_v.weight"]).view(B, T, G, d).transpose(1, 2)
        return q, k.repeat_interleave(H // G, dim=1), v.repeat_interleave(H // G, dim=1)
    if cfg.get("share_kq", False):
        bias = p["kq_bias"].to(x.dtype)
        q = F.linear(x, p["proj_q1.weight"]).unsqueeze(1) + bias[0][None, :, None, :]
        k = F.linear(x, p["proj_k1.weight"]).unsqueeze(1) + bias[1][None, :, None, :]
        v = F.linear(x, p["proj_v.weight"]).view(B, T, H, d).transpose(1, 2)
        return q, k, v
    qkv = F.linear(x, p["proj_qkv.weight"])
    q, k, v = qkv.view(B, T, 3, H, d).permute(2, 0, 3, 1, 4)
    return q, k, v


def mixer_forward(p, cfg, x, *, scan_fn=None):
    """Full mixer ``x [B,T,D] -> [B,T,D]`` (block.py:573-724), kernel or GN family.

    ``p`` maps reference state-dict names (core module, no ``_core.`` prefix,
    plus the expansion buffers) to tensors; ``cfg`` holds the core flags.
    """
    B, T, _ = x.shape
    H, d = cfg["n_heads"], cfg["head_dim"]
    eps = cfg.get("eps", 1e-6)
    q, k, v = project_qkv(p, cfg, x)
    rope = cfg.get("rope", "none")
    q = features.apply_rope(q, rope, cfg.get("rope_frac", 0.5), cfg.get("rope_base", 10000.0))
    k = features.apply_rope(k, rope, cfg.get("rope_frac", 0.5), cfg.get("rope_base", 10000.0))
    q, k = features.l2norm(q, eps), features.l2norm(k, eps)
    W1, W2 = effective_weights(p, cfg)
    log_alphas, etas = fade_parameters(p, cfg, x.dtype)
    if cfg.get("write_rule", "kernel") == "gn" and (cfg.get("depth", 1) > 1 or cfg["nonlin"] == "swiglu"
                                                     or cfg.get("write_iters", 1) == 2):
        from .gn import gn_core_net
        y = gn_core_net(q, k, v, layer_weights(p, cfg), nonlin=cfg["nonlin"],
                        learn_thresh=bool(cfg.get("learn_thresh")), read_norm=bool(cfg["read_norm"]),
                        read_norm_w1=bool(cfg.get("read_norm_w1")), write_iters=cfg.get("write_iters", 1),
                        log_alphas=log_alphas, etas=etas, mode=cfg.get("read_fade_mode", "fast"), eps=eps,
                        chunk=cfg.get("scan_chunk", 512), scan_fn=scan_fn)
    elif cfg.get("write_rule", "kernel") == "gn":
        from .gn import gn_core
        y = gn_core(q, k, v, W1, W2, p.get("Wg.0") if cfg.get("learn_thresh") else None,
                    nonlin=cfg["nonlin"], read_norm=bool(cfg["read_norm"]),
                    read_norm_w1=bool(cfg.get("read_norm_w1")), log_alphas=log_alphas, etas=etas,
                    mode=cfg.get("read_fade_mode", "fast"), eps=eps, chunk=cfg.get("scan_chunk", 512),
                    scan_fn=scan_fn)
    else:
        y = kernel_core(q, k, v, W1, W2, feature_spec(p, cfg), log_alphas=log_alphas, etas=etas,
                        mode=cfg.get("read_fade_mode", "fast"), read_norm=cfg.get("read_norm", "key_mass"),
                        eps=eps, chunk=cfg.get("scan_chunk", 512), scan_fn=scan_fn)
    if "ogate.g.lin.weight" in p:
        gate = F.linear(x, p["ogate.g.lin.weight"], p["ogate.g.lin.bias"])
        y = y * F.silu(gate.view(B, T, H, d).transpose(1, 2))
    y = y.transpose(1, 2).reshape(B, T, H * d)
    return F.linear(y, p["proj_out.weight"])
