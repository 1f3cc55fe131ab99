"""thetascan_b200 -- B200-native (sm_100a) backend for the ThetaScan mixer hot path.

Public surface (mirrors the reference package ``thetascan``):

* ``ThetaScan`` / ``ThetaScanConfig`` (+ sub-configs): the mixer module and
  its configuration, state-dict compatible with the reference;
* ``scan``: the scan-backend contract (``linattn_views`` / ``linattn``);
* ``kernel.kernel_core``: the fused kernel-family hot path;
* ``integration.install()``: register ``backend="b200"`` in an installed
  reference package.

All compute goes through the C ABI of ``include/thetascan_b200.h``.
"""
from __future__ import annotations

from .config import (GNConfig, KernelConfig, RegularizationConfig, RoPEConfig, RuntimeConfig,
                     TemporalConfig, ThetaScanConfig)
from .mixer import ThetaScan

__version__ = "0.1.0"
BACKEND_NAME = "b200"

__all__ = ["GNConfig", "KernelConfig", "RegularizationConfig", "RoPEConfig", "RuntimeConfig",
           "TemporalConfig", "ThetaScan", "ThetaScanConfig", "BACKEND_NAME"]
