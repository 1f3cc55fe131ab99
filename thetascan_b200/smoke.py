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

    # the float32 scan kernels on the same streams, within the float32 bound
    l32 = [x.float().to(device).requires_grad_(True) for x in (q, k, v)]
    outs32 = scan.linattn_views(*l32, (None, la.to(device)), append_unit=True)
    sum(o.sum() for o in outs32).backward()
    errors32 = [_rel(a, b) for a, b in zip(outs32, want)] + [_rel(a.grad, b.grad) for a, b in zip(l32, ol)]
    if max(errors32) > 1e-5:
        raise RuntimeError(f"smoke: float32 scan differs from the oracle (rel errors {errors32})")

    # the whole mixer (projections, feature kernels, scans, read) forward+backward
    _mixer(device)
    print(f"smoke ok: bf16 scan max rel err {max(errors):.2e}, float32 scan {max(errors32):.2e}")


def _mixer(device: torch.device) -> None:
    from oracle import mixer as omixer
    from .config import KernelConfig, RoPEConfig, TemporalConfig, ThetaScanConfig
    from .mixer import ThetaScan

    cfg = ThetaScanConfig(d_model=128, n_heads=2, memory_multiplier=2, feature_expansion=2, family="kernel",
                          kernel=KernelConfig(feature_map="relu2_ridge"), rope=RoPEConfig(mode="partial"),
                          temporal=TemporalConfig(mode="bank", retention_init=0.95))
    torch.manual_seed(0)
    module = ThetaScan(cfg)
    with torch.no_grad():
        gen = torch.Generator().manual_seed(1)
        module._core.W2[0].copy_(torch.randn(module._core.W2[0].shape, generator=gen) * 0.2)
    module = module.to(device)
    x = torch.randn(1, 160, 128, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16)
    xg = x.to(device).requires_grad_(True)
    y = module(xg)
    y.float().square().mean().backward()
    if _lib_status(device) != 0:
        raise RuntimeError("smoke: a kernel reported a device-side timeout")
    if not all(torch.isfinite(p.grad).all() for p in module.parameters() if p.grad is not None):
        raise RuntimeError("smoke: non-finite mixer gradient")
    core = {"n_heads": 2, "head_dim": 64, "feature_expansion": 2, "kernel_kind": "relu2_ridge", "rope": "partial",
            "rope_frac": 0.5, "rope_base": 10000.0, "read_fade": True, "read_fade_mode": "fast",
            "read_norm": "key_mass", "eps": 1e-6, "scan_chunk": 64}
    params = {n: t.detach().cpu().double() for n, t in module._core.named_parameters()}
    params.update({n: t.detach().cpu().double() for n, t in module._core.named_buffers() if n.startswith("_expand_")})
    want = omixer.mixer_forward(params, core, x.double())
    err = _rel(y, want)
    if err > 2e-2:
        raise RuntimeError(f"smoke: mixer output differs from the oracle (rel error {err:.2e})")


def _lib_status(device) -> int:
    from . import _lib
    return _lib.device_status(torch.cuda.current_stream(device).cuda_stream)
