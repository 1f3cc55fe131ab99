"""Sequence-parallel state exchange, two gloo ranks on CPU.

Each rank scans its half of the sequence from a zero state with the float64
oracle chunk scan (standing in for the GPU kernels), then applies the
exchange of :mod:`thetascan_b200.seqpar`: shard totals, an autograd
all-gather, the exclusive decayed prefix and the entering-state correction.
The corrected reads must equal the full-sequence oracle on this rank's slice,
and the gradients of q, k, v (slices) and of the log-retention (summed over
ranks) must equal the full-sequence gradients.  Tolerance 1e-10 (float64).
"""
from __future__ import annotations

import datetime
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import scan as oscan

WORLD = 2
B, H, T, DK, DV, CHUNK = 1, 2, 96, 12, 5, 16


def _inputs():
    g = torch.Generator().manual_seed(11)
    q = torch.rand(B, H, T, DK, generator=g, dtype=torch.float64)
    k = torch.rand(B, H, T, DK, generator=g, dtype=torch.float64)
    v = torch.randn(B, H, T, DV, generator=g, dtype=torch.float64)
    la = torch.log(0.9 + 0.09 * torch.rand(H, generator=g, dtype=torch.float64))
    w = [torch.randn(B, H, T, DV + 1, generator=g, dtype=torch.float64) for _ in range(2)]
    return q, k, v, la, w


def _aug(v):
    return torch.cat((v, torch.ones(*v.shape[:-1], 1, dtype=v.dtype)), dim=-1)


def _full_reference():
    q, k, v, la, w = _inputs()
    leaves = [t.clone().requires_grad_(True) for t in (q, k, v, la)]
    outs = oscan.linattn_chunk_views(leaves[0], leaves[1], _aug(leaves[2]), (None, leaves[3]), CHUNK)
    loss = sum((o * wr).sum() for o, wr in zip(outs, w))
    loss.backward()
    return [o.detach() for o in outs], [t.grad for t in leaves]


def _worker(rank, port, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=60))
    try:
        from thetascan_b200 import seqpar
        q, k, v, la, w = _inputs()
        L = T // WORLD
        sl = slice(rank * L, (rank + 1) * L)
        qs, ks, vs = (t[:, :, sl].clone().requires_grad_(True) for t in (q, k, v))
        las = [None, la.clone().requires_grad_(True)]
        local = oscan.linattn_chunk_views(qs, ks, _aug(vs), tuple(las), CHUNK)
        slots = seqpar.exchange(seqpar.nccl_shard(), las)(qs, ks, vs, list(local))
        loss = sum((o * wr[:, :, sl]).sum() for o, wr in zip(slots, w))
        loss.backward()
        dla = las[1].grad.clone()
        dist.all_reduce(dla)
        torch.save({"slots": [o.detach() for o in slots], "dq": qs.grad, "dk": ks.grad, "dv": vs.grad,
                    "dla": dla}, os.path.join(out_dir, f"rank{rank}.pt"))
        dist.barrier()   # both ranks done with every collective before teardown
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_rank_exchange_matches_full_sequence(tmp_path):
    mp.spawn(_worker, args=(_free_port(), str(tmp_path)), nprocs=WORLD, join=True)
    outs, grads = _full_reference()
    L = T // WORLD
    for rank in range(WORLD):
        got = torch.load(tmp_path / f"rank{rank}.pt")
        sl = slice(rank * L, (rank + 1) * L)
        for o_got, o_ref in zip(got["slots"], outs):
            assert torch.allclose(o_got, o_ref[:, :, sl], rtol=1e-10, atol=1e-10)
        for name, ref in zip(("dq", "dk", "dv"), grads[:3]):
            assert torch.allclose(got[name], ref[:, :, sl], rtol=1e-10, atol=1e-10), name
        assert torch.allclose(got["dla"], grads[3], rtol=1e-9, atol=1e-10)


def test_sequential_shards_match_full_sequence():
    """The single-process stand-in runs the shards in order in one graph."""
    from thetascan_b200 import seqpar
    q, k, v, la, w = _inputs()
    P, L = 3, T // 3
    leaves = [t.clone().requires_grad_(True) for t in (q, k, v, la)]
    runner = seqpar.SequentialShards(P)
    pieces = []
    for rank in range(P):
        sl = slice(rank * L, (rank + 1) * L)
        qs, ks, vs = (t[:, :, sl] for t in leaves[:3])
        las = [None, leaves[3]]
        local = oscan.linattn_chunk_views(qs, ks, _aug(vs), tuple(las), CHUNK)
        pieces.append(seqpar.exchange(runner.shard(rank), las)(qs, ks, vs, list(local)))
    outs = [torch.cat([p[r] for p in pieces], dim=2) for r in range(2)]
    loss = sum((o * wr).sum() for o, wr in zip(outs, w))
    loss.backward()
    ref_outs, ref_grads = _full_reference()
    for o_got, o_ref in zip(outs, ref_outs):
        assert torch.allclose(o_got, o_ref, rtol=1e-10, atol=1e-10)
    for got, ref in zip(leaves, ref_grads):
        assert torch.allclose(got.grad, ref, rtol=1e-9, atol=1e-10)


def _gn_worker(rank, port, out_dir, name):
    """One rank of a two-rank GN mixer: its half of the sequence through the
    deep / swiglu GN core, every read exchanging shard totals with the other
    rank over the gloo group (several all-gathers per forward and their
    backward collectives)."""
    import sys
    import types
    sys.path.insert(0, os.path.dirname(__file__))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=60))
    try:
        import test_gn_deep_host as host
        from thetascan_b200 import gn_deep, seqpar
        from thetascan_b200.config import ThetaScanConfig
        from thetascan_b200.mixer import ThetaScan
        gn_deep._scan = types.SimpleNamespace(linattn_views=host.oracle_views)
        case = torch.load(os.path.join(host.GOLDEN, "gn_deep_cases.pt"), weights_only=False)[name]
        cfg = ThetaScanConfig.from_dict(case["public_config"])
        module = ThetaScan(cfg)
        module.load_state_dict({"_core." + n: t.float() for n, t in case["params"].items()
                                if not n.startswith("_expand_")})
        L = case["x"].shape[1] // WORLD
        sl = slice(rank * L, (rank + 1) * L)
        x = case["x"][:, sl].float().clone().requires_grad_(True)
        y = host._mixer(module._core, cfg, x, seqpar.nccl_shard())
        (y.double() * case["out_weight"][:, sl]).sum().backward()
        grads = {n: p.grad.clone() for n, p in module._core.named_parameters() if p.grad is not None}
        for g in grads.values():
            dist.all_reduce(g)
        torch.save({"y": y.detach(), "x_grad": x.grad, "grads": grads}, os.path.join(out_dir, f"gn{rank}.pt"))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_rank_gn_shards_match_reference_fixture(tmp_path):
    """A depth-2 swiglu GN mixer with a stale bank on two gloo ranks: the
    concatenated outputs, the input gradient and the rank-summed parameter
    gradients equal the reference's unsharded fixture (float32 per-token
    maps, 1e-4)."""
    name = "gn_depth2_swiglu_stale"
    mp.spawn(_gn_worker, args=(_free_port(), str(tmp_path), name), nprocs=WORLD, join=True)
    case = torch.load(os.path.join(os.path.dirname(__file__), "golden", "gn_deep_cases.pt"),
                      weights_only=False)[name]
    got = [torch.load(tmp_path / f"gn{r}.pt") for r in range(WORLD)]

    def rel(a, b):
        return float((a.double() - b.double()).abs().max() / b.double().abs().max())

    assert rel(torch.cat([g["y"] for g in got], dim=1), case["y"]) < 1e-4
    assert rel(torch.cat([g["x_grad"] for g in got], dim=1), case["x_grad"]) < 1e-4
    for n, want in case["grads"].items():
        assert rel(got[0]["grads"][n], want) < 1e-4, n
