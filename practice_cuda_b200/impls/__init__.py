"""Importing this package registers the sm_100a implementations.

Names: ``b200_per_block_{1d,2d}``, ``b200_per_block_1x128_128x128`` (1x128
activation tiles with 128x128 weight tiles), ``b200_per_block_e8m0_1x128_128x128``
(the same with power-of-two scales on the block-scaled GEMM), ``b200_per_channel``,
``b200_per_channel_one_pass``, ``b200_per_tensor`` and their BMM layouts.  The
reference's names (``triton_per_block_1d_a_k_b_n``, ...) are registered as
aliases of the same functions, so harness code that looks up the reference
names runs on these kernels unchanged.
"""

from . import b200_per_block as _b200_per_block
from . import b200_per_channel as _b200_per_channel
from . import b200_per_tensor as _b200_per_tensor

for _prefix in ("b200", "triton"):
    _b200_per_block.register_all(_prefix)
    _b200_per_channel.register_all(_prefix)
    _b200_per_tensor.register_all(_prefix)

# 1x128 activation tiles with 128x128 weight tiles (DeepSeek-V3 style); the
# quant impl registered under this name quantizes with the A-side blocks.
_b200_per_block._register_block_scheme(
    "b200_per_block_1x128_128x128",
    a_block=(1, 128),
    b_block=(128, 128),
    description="1x128 activation blocks with 128x128 weight blocks.",
)
# The same tiles with power-of-two (E8M0) scales: the BMM layouts run the
# block-scaled tensor-core GEMM (not a reference scheme; the FP8 training recipe).
_b200_per_block._register_block_scheme(
    "b200_per_block_e8m0_1x128_128x128",
    a_block=(1, 128),
    b_block=(128, 128),
    description="1x128 / 128x128 blocks with power-of-two scales applied by the tensor core.",
    pow2_scales=True,
)

__all__ = []
