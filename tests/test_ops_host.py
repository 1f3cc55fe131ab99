"""The ``thetascan_b200`` custom operators on the host (no GPU): every op is
registered with a schema, the forward ops have fake implementations whose
workspace size is the C ABI's own answer, and CPU tensors are refused with
``RuntimeError`` before anything reaches the library (no CPU fallback)."""
from __future__ import annotations

import pytest
import torch

from thetascan_b200 import ops

NAMES = ["scan_views_fwd", "scan_views_bwd", "kernel_mixer_fwd", "kernel_mixer_bwd", "kernel_mixer_qkv_fwd",
         "kernel_mixer_qkv_bwd", "scan_views_stream_fwd", "scan_views_stream_bwd"]


@pytest.mark.parametrize("name", NAMES)
def test_op_is_registered(name):
    op = getattr(torch.ops.thetascan_b200, name)
    assert op.default._schema.name == f"thetascan_b200::{name}"


def test_cpu_tensors_raise_like_the_reference_cuda_backends():
    q = torch.zeros(1, 2, 8, 4)
    with pytest.raises(RuntimeError, match="CUDA"):
        torch.ops.thetascan_b200.scan_views_fwd(q, q, q, [], [False], 1, [False], False)
    W1, W2 = torch.zeros(2, 16, 4), torch.zeros(2, 4, 16)
    with pytest.raises(RuntimeError, match="CUDA"):
        torch.ops.thetascan_b200.kernel_mixer_fwd(q.bfloat16(), q.bfloat16(), q.bfloat16(), W1, W2, None, None,
                                                  None, None, None, None, None, None, "relu2_ridge", "sum", 1e-6,
                                                  8.0, 8, 3.0, 1.0, "none", 0.25)


def test_fake_workspace_is_the_library_size_query():
    # config-2 shape of one head: m = 256 features, payload [v | 1 | 1], two slots
    n = ops._scan_workspace_nbytes(1, 1, 4096, 256, 64, 2, [False, True], [False, False], False)
    nt, dkm, dvp, dkp = 32, 256, 80, 256
    states = nt * 2 * dkm * dvp * 4
    images = nt * 2 * dvp * dkp * 2
    assert n == states + images
