"""CPU oracle for the FP8 quantize / scaled-BMM path.

TEST INFRASTRUCTURE ONLY.  Nothing in ``practice_cuda_b200`` imports this
package: it is the checker used by ``tests/``, ``__graft_entry__.smoke()`` and
the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py``.  The product
path runs the CUDA library and fails loudly when it is missing.

Parity pin: the restatement is checked against vectors produced by the
reference's own torch functions (``tests/golden/make_golden.py``) -- the
per-channel torch quantizer, the legacy per-tensor test reference, and the
registry's ``QuantResult.dequantize``, and the FP8 training linear's dynamic
cast ``hp_tensor_to_float8_dynamic``.
"""

from .quant import (  # noqa: F401
    FP8_MAX,
    per_block_quant,
    per_block_quant_pow2,
    per_channel_quant,
    per_tensor_quant,
    legacy_per_tensor_quant,
    float8_dynamic_cast,
    dequantize,
)
from .gemm import (  # noqa: F401
    scaled_bmm_dequant_reference,
    scaled_bmm_promoted_reference,
    legacy_bmm_reference,
)
