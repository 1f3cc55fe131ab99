"""Scan-level oracles: inclusive causal linear attention with scalar retention.

Contract (reference ``src/thetascan/_core/ops/scan_chunk.py:246-268``):
``out[t] = sum_{i<=t} w(t, i) * (q_t . k_i) * v_i`` for ``q, k`` of shape
``[B, H, T, Dk]`` and ``v`` of shape ``[B, H, T, Dv]``.  A retention is either
``None`` (plain causal sum, ``w = 1``), a static per-head log-retention of
shape ``[H]`` (``w = alpha_h^(t-i)``) or a per-token scalar log-retention
stream of shape ``[B, H, T, 1]`` (``w = exp(sum_{i<s<=t} la_s)``).

These are test infrastructure only (see the package docstring).
"""
from __future__ import annotations

import torch

# Guard of the reference prefix-sum backend (scan_cumsum.py:4).
CUMSUM_CLAMP = 60.0


def _as_stream(retention: torch.Tensor | None, like: torch.Tensor) -> torch.Tensor | None:
    """Widen a static ``[H]`` retention to ``[B,H,T,1]``.

    Follows ``interface._retention_stream`` (interface.py:110-117).
    """
    if retention is None or retention.ndim == 4:
        return retention
    B, H, T = like.shape[:3]
    return retention.to(like.dtype).reshape(1, H, 1, 1).expand(B, H, T, 1)


def linattn_naive(q, k, v, decay=None):
    """Sequential recurrence S <- alpha*S + k v^T; out = q^T S.

    Restates ``scan_naive.linattn`` (scan_naive.py:5-18), including the
    per-key-channel decay form ``[B,H,T,Dk]``.
    """
    B, H, T, Dk = k.shape
    state = q.new_zeros(B, H, Dk, v.shape[-1])
    rows = []
    for t in range(T):
        if decay is not None:
            state = state * decay[:, :, t].exp().unsqueeze(-1)
        state = state + k[:, :, t, :, None] * v[:, :, t, None, :]
        rows.append(torch.einsum("bhk,bhkv->bhv", q[:, :, t], state))
    return torch.stack(rows, dim=2)


def linattn_quad(q, k, v, decay=None):
    """Masked ``[T,T]`` dual form (scan_quad.py:5-16)."""
    T = q.shape[2]
    scores = q @ k.transpose(-1, -2)
    if decay is not None:
        if decay.shape[-1] != 1:
            raise NotImplementedError("quad oracle: scalar decay only")
        cum = decay[..., 0].cumsum(-1)
        scores = scores * (cum[..., :, None] - cum[..., None, :]).clamp(max=0.0).exp()
    causal = torch.ones(T, T, dtype=torch.bool, device=q.device).tril()
    return scores.masked_fill(~causal, 0.0) @ v


def linattn_cumsum(q, k, v, decay=None):
    """Materialised prefix-sum form (scan_cumsum.py:7-19).

    ``S_t = cumsum(k (x) v)`` of shape ``[B,H,T,Dk,Dv]``; a decay divides by a
    clamped cumulative product.  This is the reference's CPU baseline arm; it is
    numerically invalid once ``sum(log alpha) < -60`` (the reference says so).
    """
    if decay is None:
        states = (k.unsqueeze(-1) * v.unsqueeze(-2)).cumsum(2)
        return torch.einsum("bhtk,bhtkv->bhtv", q, states)
    if decay.shape[-1] != 1:
        raise NotImplementedError("cumsum oracle: scalar decay only")
    cum = decay[..., 0].cumsum(-1)
    grow = (-cum).clamp(max=CUMSUM_CLAMP).exp().unsqueeze(-1)
    states = ((k * grow).unsqueeze(-1) * v.unsqueeze(-2)).cumsum(2)
    out = torch.einsum("bhtk,bhtkv->bhtv", q, states)
    return out * cum.clamp(min=-CUMSUM_CLAMP).exp().unsqueeze(-1)


def _tile_log_phases(retention, B, H, T, width, tiles, dtype):
    """Per-position cumulative log-retention local to each tile, ``[B,H,NT,C]``.

    Static retentions use the exact product ``(i+1) * la`` and streams the
    tile-local cumulative sum, mirroring ``_static_weights`` /
    ``_tile_weights`` (scan_chunk.py:102-155).  Phases are formed in at least
    float32 (scan_chunk.py:89-99).
    """
    phase = torch.float64 if dtype == torch.float64 else torch.float32
    if retention.ndim == 4:
        padded = torch.zeros(B, H, tiles * width, dtype=phase)
        padded[:, :, :T] = retention[..., 0].to(phase)
        return padded.view(B, H, tiles, width).cumsum(-1)
    index = torch.arange(width, dtype=phase) + 1.0
    la = retention.to(phase).reshape(1, H, 1, 1)
    return (la * index).expand(B, H, tiles, width)


def linattn_chunk_views(q, k, v, retentions, chunk: int = 512):
    """Chunked scan of one stream set through several retentions at once.

    Restates ``scan_chunk.linattn_views`` (scan_chunk.py:246-339): one score
    tile per chunk shared by every view, an intra-tile retention weight
    ``exp(min(L_i - L_j, 0))`` on the causal triangle, an exclusive carried
    state promoted to at least float32 (scan_chunk.py:301), the carry weight
    ``exp(L_i)`` on the cross term and the closing weight ``exp(L_{C-1})`` on
    the state (scan_chunk.py:326-336).  Errors follow scan_chunk.py:269-290.
    """
    if chunk < 1:
        raise ValueError("chunk backend: chunk must be >= 1")
    if not retentions:
        return ()
    B, H, T = q.shape[:3]
    for retention in retentions:
        if retention is None:
            continue
        if retention.ndim == 4:
            if retention.shape[-1] != 1:
                raise NotImplementedError("chunk backend: scalar decay only (v1)")
        elif retention.numel() != H:
            raise ValueError(
                "chunk backend: a static retention needs one entry per head, "
                f"got {tuple(retention.shape)} for q {tuple(q.shape)}"
            )
    width = min(chunk, T)
    tiles = -(-T // width)
    pad = tiles * width - T
    state_dtype = torch.promote_types(q.dtype, torch.float32)

    def tiled(x):
        if pad:
            x = torch.cat([x, x.new_zeros(*x.shape[:2], pad, *x.shape[3:])], dim=2)
        return x.view(B, H, tiles, width, x.shape[-1])

    qt, kt, vt = tiled(q), tiled(k), tiled(v)
    scores = qt @ kt.transpose(-1, -2)
    causal = torch.ones(width, width, dtype=torch.bool).tril()
    outputs = []
    for retention in retentions:
        if retention is None:
            weight = None
        else:
            L = _tile_log_phases(retention, B, H, T, width, tiles, q.dtype)
            weight = (L[..., :, None] - L[..., None, :]).clamp(max=0.0).exp()
        masked = scores if weight is None else scores * weight.to(q.dtype)
        intra = masked.masked_fill(~causal, 0.0) @ vt
        state = q.new_zeros(B, H, q.shape[-1], v.shape[-1], dtype=state_dtype)
        cross = []
        for n in range(tiles):
            kn, vn = kt[:, :, n], vt[:, :, n]
            read = qt[:, :, n] @ state.to(q.dtype)
            if weight is None:
                cross.append(read)
                update = kn.transpose(-1, -2).to(state_dtype) @ vn.to(state_dtype)
                state = state + update
            else:
                Ln = L[:, :, n]
                cross.append(read * Ln.exp().to(q.dtype).unsqueeze(-1))
                keyed = kn * (Ln[..., -1:] - Ln).exp().to(q.dtype).unsqueeze(-1)
                update = keyed.transpose(-1, -2).to(state_dtype) @ vn.to(state_dtype)
                state = state * Ln[..., -1].exp().to(state_dtype)[..., None, None] + update
        out = intra + torch.stack(cross, dim=2)
        outputs.append(out.reshape(B, H, tiles * width, -1)[:, :, :T])
    return tuple(outputs)


def linattn_chunk(q, k, v, decay=None, chunk: int = 512, log_alpha=None):
    """One-view wrapper (scan_chunk.py:342-358); ``log_alpha`` wins."""
    retention = log_alpha if log_alpha is not None else decay
    return linattn_chunk_views(q, k, v, (retention,), chunk)[0]


def ema_cumsum(x, log_alpha, chunk: int = 64):
    """Static-retention discounted prefix ``z_t = sum_{i<=t} alpha^(t-i) x_i``.

    Restates ``interface.ema_cumsum`` (interface.py:58-93) through the scan
    identity: a unit query/key scan of the payload ``x``.
    """
    ones = x.new_ones(*x.shape[:3], 1)
    return linattn_chunk_views(ones, ones, x, (log_alpha,), chunk)[0]


def causal_prefix_sum(x):
    """Plain prefix along T (interface.py:96-107)."""
    return x.cumsum(2)
