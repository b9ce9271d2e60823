"""practice_cuda_b200: the FP8 quantize / scaled-BMM hot path of
xuOAO/practice_cuda, rebuilt for B200 (sm_100a).

Kernels live in libpcb200.so (``csrc/``, C ABI in ``include/pcb200.h``);
this package is the host side that mirrors the reference's plugin registry
(``registry``), its impl modules (``impls``) and legacy entry points
(``fp8_warper``).
"""

from .registry import (  # noqa: F401
    BMM_IMPLS,
    QUANT_IMPLS,
    BMMImpl,
    QuantImpl,
    QuantResult,
    bmm_impl_names,
    get_bmm,
    get_quant,
    load_builtin_impls,
    register_bmm,
    register_quant,
)

__version__ = "0.1.0"
