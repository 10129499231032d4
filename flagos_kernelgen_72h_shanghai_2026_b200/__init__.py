"""B200-native fused residual-add + RMSNorm + per-token group quantisation.

Drop-in for ``fused_add_rmsnorm_group_quant`` of
sinpeyw/flagos-kernelgen-72h-shanghai-2026
(src/task01_fused_add_rmsnorm_group_quant.py:1731-1851): same positional
signature, destination passing, same returned tensor objects. The device
work is one hand-written sm_100a kernel in libfarq.so (C ABI: include/farq.h).
"""
from .offload import fused_add_rmsnorm_group_quant_host  # noqa: F401
from .task01 import fused_add_rmsnorm_group_quant, launch_plan  # noqa: F401

__all__ = ["fused_add_rmsnorm_group_quant", "fused_add_rmsnorm_group_quant_host", "launch_plan"]
