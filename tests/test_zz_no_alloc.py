"""The allocation-free scan entry point (``ts_b200_scan_fwd_static``).

Some hosts cannot allocate device memory for a plug-in: their allocator owns
all of it, or they forbid cudaMalloc once serving.  For them the library keeps
its scan scratch in a fixed device array.  These tests call that entry point
through the C ABI, twice in a row with different inputs, and check each result
against the workspace entry point (``ts_b200_scan_fwd``) within the parity
tolerance of the GPU tests; then they check that an oversized shape is refused
before anything is launched.  The file is collected last so that a failure
here never hides the other GPU tests.
"""
from __future__ import annotations

import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu
BF16_TOL = 2e-2


def _rel(got, want):
    got, want = got.double().cpu(), want.double().cpu()
    return float((got - want).abs().max() / want.abs().max().clamp_min(1e-30))


def _inputs(seed, B=2, H=2, T=600, Dk=64, Dv=64):
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(B, H, T, Dk, generator=g) / math.sqrt(Dk)).abs().to(torch.bfloat16).cuda()
    k = (torch.randn(B, H, T, Dk, generator=g) / math.sqrt(Dk)).abs().to(torch.bfloat16).cuda()
    v = torch.randn(B, H, T, Dv, generator=g).to(torch.bfloat16).cuda()
    la = torch.log(0.85 + 0.14 * torch.rand(H, generator=g)).float().cuda()
    return q, k, v, la


def _run(lib, scan, fn_name, q, k, v, la, workspace):
    outs = [torch.empty(*q.shape[:3], v.shape[-1] + 1, dtype=torch.float32, device="cuda") for _ in range(2)]
    args = scan._build_args(q, k, v, [None, la], outs, True)
    if workspace:
        nbytes = lib.load().ts_b200_scan_workspace_bytes(ctypes.byref(args))
        ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
        args.workspace, args.workspace_bytes = ws.data_ptr(), ws.numel()
    lib.check(getattr(lib.load(), fn_name)(ctypes.byref(args), scan._stream()))
    assert lib.device_status(torch.cuda.current_stream().cuda_stream) == 0
    return outs


@pytest.fixture(scope="module")
def mods():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from thetascan_b200 import _lib, scan
    return _lib, scan


def test_static_scratch_matches_workspace_entry_point_twice(mods):
    lib, scan = mods
    for seed, T in ((11, 600), (12, 333)):
        q, k, v, la = _inputs(seed, T=T)
        got = _run(lib, scan, "ts_b200_scan_fwd_static", q, k, v, la, workspace=False)
        want = _run(lib, scan, "ts_b200_scan_fwd", q, k, v, la, workspace=True)
        for a, b in zip(got, want):
            assert _rel(a, b) <= BF16_TOL


def test_static_scratch_rejects_oversized_shapes(mods):
    lib, scan = mods
    q, k, v, la = _inputs(13, B=1, H=1, T=128)
    outs = [torch.empty(1, 1, 128, 65, device="cuda") for _ in range(2)]
    args = scan._build_args(q, k, v, [None, la], outs, True)
    # Declare a shape whose states exceed the fixed scratch: refused on the
    # host before any launch, so the small buffers above are never touched.
    args.batch, args.heads, args.tokens = 64, 16, 1 << 16
    rc = lib.load().ts_b200_scan_fwd_static(ctypes.byref(args), scan._stream())
    assert rc == lib.TS_ERR_VALUE
    assert "static scratch" in lib.last_error()[1]
