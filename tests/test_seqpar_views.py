"""Sequence shards of any view on CPU: ``seqpar.sharded_reads``.

The shards of a sequence run one after another (``SequentialShards``), each
reading its tokens from a zero state with the float64 oracle scan and taking
the earlier shards' state through the exchange; concatenated, their reads
must equal the reads of the whole sequence -- plain sum, decayed and stale
views, with and without the unit column -- and so must the gradients of the
streams and of the log-retentions (float64, 1e-10).
"""
from __future__ import annotations

import pytest
import torch

from oracle import scan as oracle_scan
from thetascan_b200 import seqpar


def oracle_views(q, k, v, retentions, chunk=512, *, append_unit=False, stale=None):
    stale = stale or (False,) * len(retentions)
    if append_unit:
        v = torch.cat([v, v.new_ones(*v.shape[:3], 1)], dim=-1)
    outs = oracle_scan.linattn_chunk_views(q, k, v, tuple(retentions) + (None,), 16)
    return tuple(outs[-1] - o if st else o for o, st in zip(outs[:-1], stale))


@pytest.mark.parametrize("append_unit", [False, True])
@pytest.mark.parametrize("P", [2, 3])
def test_sharded_reads_equal_whole_sequence(P, append_unit):
    g = torch.Generator().manual_seed(P)
    B, H, T, dk, dv = 2, 2, 48 * P, 8, 5
    q, k, v = (torch.randn(B, H, T, n, generator=g, dtype=torch.float64).requires_grad_(True)
               for n in (dk, dk, dv))
    la = (-torch.rand(H, generator=g, dtype=torch.float64) * 0.2).requires_grad_(True)
    rets, stale = (None, la, la), (False, False, True)
    want = oracle_views(q, k, v, rets, append_unit=append_unit, stale=stale)
    w = [torch.randn(o.shape, generator=g, dtype=torch.float64) for o in want]
    grads_want = torch.autograd.grad(sum((o * wi).sum() for o, wi in zip(want, w)), (q, k, v, la))

    runner = seqpar.SequentialShards(P)
    L = T // P
    pieces = [[] for _ in rets]
    for p in range(P):
        sl = slice(p * L, (p + 1) * L)
        out = seqpar.sharded_reads(runner.shard(p), oracle_views, q[:, :, sl], k[:, :, sl], v[:, :, sl], rets,
                                   append_unit=append_unit, stale=stale)
        for i, o in enumerate(out):
            pieces[i].append(o)
    got = [torch.cat(ps, dim=2) for ps in pieces]
    for a, b in zip(got, want):
        assert (a - b).abs().max() / b.abs().max() < 1e-10
    grads_got = torch.autograd.grad(sum((o * wi).sum() for o, wi in zip(got, w)), (q, k, v, la))
    for a, b in zip(grads_got, grads_want):
        assert (a - b).abs().max() / b.abs().max() < 1e-10


def test_sequential_shards_keep_exchanges_apart():
    runner = seqpar.SequentialShards(2)
    s0 = runner.shard(0)
    a0, b0 = torch.ones(3), 2 * torch.ones(3)
    assert s0.gather(a0)[0] is a0 and s0.gather(b0)[0] is b0
    s1 = runner.shard(1)
    first = s1.gather(torch.zeros(3))
    second = s1.gather(torch.zeros(3))
    assert first[0] is a0 and second[0] is b0
    with pytest.raises(ValueError):
        runner.shard(3)


def test_float32_shard_views_cut_wide_payloads(monkeypatch):
    """The float32 kernel-family path's sharded reads (``precise._views_fn``)
    cut payloads wider than the float32 scan kernels take (256 columns with
    the exchange's unit column) into pieces; around the oracle scan, the
    pieces of a 300-column payload with the unit column equal the whole
    sequence's read."""
    from thetascan_b200 import precise
    monkeypatch.setattr(precise, "linattn_views", oracle_views)
    g = torch.Generator().manual_seed(3)
    B, H, T, P = 1, 2, 64, 2
    q, k = (torch.rand(B, H, T, 1, generator=g, dtype=torch.float64) for _ in range(2))
    v = torch.randn(B, H, T, 300, generator=g, dtype=torch.float64)
    la = -torch.rand(H, generator=g, dtype=torch.float64) * 0.1
    rets, stale = (None, la), (False, True)
    want = oracle_views(q, k, v, rets, append_unit=True, stale=stale)
    runner = seqpar.SequentialShards(P)
    L = T // P
    parts = [precise._views_fn(runner.shard(p))(q[:, :, p * L:(p + 1) * L], k[:, :, p * L:(p + 1) * L],
                                               v[:, :, p * L:(p + 1) * L], rets, append_unit=True, stale=stale)
             for p in range(P)]
    for i, w in enumerate(want):
        got = torch.cat([pt[i] for pt in parts], dim=2)
        assert got.shape == w.shape
        assert (got - w).abs().max() / w.abs().max() < 1e-10
