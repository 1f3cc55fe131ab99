"""Smoke check used by ``__graft_entry__.smoke``: one small forward+backward of
the hot path on a CUDA device, compared with the float64 CPU oracle.

The oracle is imported lazily and only here (a checker, never the thing run).
"""
from __future__ import annotations

import math

import torch


def _rel(got, want):
    got = got.detach().to("cpu", torch.float64)
    want = want.detach().to("cpu", torch.float64)
    return float((got - want).abs().max() / want.abs().max().clamp_min(1e-30))


def run(device: torch.device) -> None:
    from oracle import scan as oscan
    from . import _lib, scan

    g = torch.Generator().manual_seed(0)
    B, H, T, Dk, Dv = 1, 2, 300, 64, 64
    q = (torch.randn(B, H, T, Dk, generator=g) / math.sqrt(Dk)).to(torch.bfloat16)
    k = (torch.randn(B, H, T, Dk, generator=g) / math.sqrt(Dk)).to(torch.bfloat16)
    v = torch.randn(B, H, T, Dv, generator=g).to(torch.bfloat16)
    la = torch.log(torch.tensor([0.9, 0.99]))
    leaves = [x.to(device).requires_grad_(True) for x in (q, k, v)]
    outs = scan.linattn_views(*leaves, (None, la.to(device)), append_unit=True)
    sum(o.float().sum() for o in outs).backward()
    if _lib.device_status(torch.cuda.current_stream(device).cuda_stream) != 0:
        raise RuntimeError("smoke: a kernel reported a device-side timeout")
    ol = [x.double().requires_grad_(True) for x in (q, k, v)]
    unit = torch.cat([ol[2], torch.ones_like(ol[2][..., :1])], dim=-1)
    want = oscan.linattn_chunk_views(ol[0], ol[1], unit, (None, la.double()), chunk=128)
    sum(o.sum() for o in want).backward()
    errors = [_rel(a, b) for a, b in zip(outs, want)]
    errors += [_rel(a.grad, b.grad) for a, b in zip(leaves, ol)]
    if max(errors) > 2e-2:
        raise RuntimeError(f"smoke: CUDA path differs from the oracle (rel errors {errors})")
    print(f"smoke ok: max rel err {max(errors):.2e}")
