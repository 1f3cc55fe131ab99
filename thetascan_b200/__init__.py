"""thetascan_b200 -- B200-native (sm_100a) backend for the ThetaScan mixer hot path.

The package exposes the reference's scan-backend interface (``scan``: the
``linattn_views`` / ``linattn`` contract of the reference chunk backend) on top
of hand-written tcgen05 kernels reached through the C ABI declared in
``include/thetascan_b200.h``.
"""
from __future__ import annotations

__version__ = "0.1.0"

BACKEND_NAME = "b200"
