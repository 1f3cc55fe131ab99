"""CPU oracle for the ThetaScan mixer hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in float64 PyTorch on the CPU, the algorithms of the
reference ThetaScan v0.1.0 hot path: the causal linear-attention scans
(sequential, masked dual form, prefix-sum and chunked forms), the positive
kernel feature maps, the key-mass normalized read with its temporal views, and
the kernel-family mixer that composes them.  Every function cites the
reference ``file:line`` it follows (paths are relative to the reference
project root).

Who may use it: only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py``, and there only as
the checker or as the timed CPU baseline.  The product (``thetascan_b200``)
never imports anything from here; its CUDA path fails loudly when its
extension is missing instead of falling back to this code.

Parity pinning: ``tests/golden/make_golden.py`` imports the real reference
package in the build container and records its outputs and gradients as small
fixtures under ``tests/golden/``; ``tests/test_oracle_golden.py`` checks this
oracle against those fixtures (float64, rtol 1e-9), so the oracle is pinned to
the reference, not only to itself.
"""
