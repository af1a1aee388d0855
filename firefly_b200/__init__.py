"""firefly_b200 — FireFly's INT8 training hot path, native to NVIDIA B200 (sm_100a).

Drop-in for the reference package's public API (fumitoshi0524/FireFly
``__init__.py:1-10``): ``BitLinear``, ``FireFlyOptim``,
``collect_bitlinear_modules``, ``quantize_fp_to_int8``.  The compute runs in
libfirefly_b200.so (hand-written sm_100a kernels) through a C ABI
(``include/firefly_b200.h``).
"""
from .fireflykernels import quantize_fp_to_int8
from .bitLinear import BitLinear, collect_bitlinear_modules
from .fireflyoptim import FireFlyOptim, FireFlyOptimSR

__all__ = [
    "BitLinear",
    "FireFlyOptim",
    "FireFlyOptimSR",
    "collect_bitlinear_modules",
    "quantize_fp_to_int8",
]
