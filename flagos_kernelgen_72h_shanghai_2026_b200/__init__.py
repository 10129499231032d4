"""B200-native fused residual-add + RMSNorm + per-token group quantisation.

Drop-in for ``fused_add_rmsnorm_group_quant`` of
sinpeyw/flagos-kernelgen-72h-shanghai-2026
(src/task01_fused_add_rmsnorm_group_quant.py:1731-1851): same positional
signature, destination passing, same returned tensor objects. The device
work is one hand-written sm_100a kernel in libfarq.so (C ABI: include/farq.h).

Also a drop-in for ``dsa_topk_page_table_transform``
(src/task02_dsa_topk_page_table_transform.py:1666): one sm_100a kernel in
libdsa_topk.so (C ABI: include/dsa_topk.h).
"""
from .offload import fused_add_rmsnorm_group_quant_host  # noqa: F401
from .task01 import fused_add_rmsnorm_group_quant, launch_plan  # noqa: F401
from .task02 import dsa_topk_page_table_transform  # noqa: F401
from . import task01, task02  # noqa: F401,E402

__all__ = ["fused_add_rmsnorm_group_quant", "fused_add_rmsnorm_group_quant_host", "launch_plan",
           "dsa_topk_page_table_transform"]
