"""Legacy entry points of ``kernels/fp8_bmm`` with their signatures kept.

``fp8_quant_triton`` (``kernels/fp8_bmm/fp8_warper.py:9-77``) and
``fp8_bmm_quant_triton`` (:79-129) plus ``FP8Format``
(``kernels/fp8_bmm/fp8_utils.py:11-31``), running on libpcb200.
"""

from __future__ import annotations

from enum import Enum
from typing import NamedTuple

import torch

from . import _lib
from .impls._common import bmm_scaled
from .impls.b200_per_tensor import quantize_per_tensor


class _FormatHelper(NamedTuple):
    max_fwd: float
    max_bwd: float
    dtype_fwd: torch.dtype
    dtype_bwd: torch.dtype


class FP8Format(Enum):
    E4M3 = _FormatHelper(max_fwd=448.0, max_bwd=448.0, dtype_fwd=torch.float8_e4m3fn,
                         dtype_bwd=torch.float8_e4m3fn)
    E5M2 = _FormatHelper(max_fwd=57344.0, max_bwd=57344.0, dtype_fwd=torch.float8_e5m2,
                         dtype_bwd=torch.float8_e5m2)
    HYBRID = _FormatHelper(max_fwd=448.0, max_bwd=57344.0, dtype_fwd=torch.float8_e4m3fn,
                           dtype_bwd=torch.float8_e5m2)


def fp8_quant_triton(
    x: torch.Tensor,
    quant_dtype=FP8Format.E4M3.value.dtype_fwd,
    fp8_range=FP8Format.E4M3.value.max_fwd,
    eps=1e-12,
    is_test=False,
):
    """Per-tensor quantization; returns ``(fp8 tensor, reciprocal factor)``.

    As in the reference, the scale arithmetic runs in ``x``'s dtype and the
    reciprocal factor is a 0-dim tensor of that dtype.  ``is_test`` only chose
    a Triton kernel variant and is accepted for compatibility.
    """
    del is_test
    if isinstance(quant_dtype, FP8Format):
        quant_dtype = quant_dtype.value.dtype_fwd
    if x.dim() not in (2, 3):
        raise RuntimeError("dim must eq 2 or 3")
    quanted_x, _, recip = quantize_per_tensor(x, quant_dtype, float(fp8_range), eps, scale_dtype=x.dtype)
    return quanted_x, recip.to(x.dtype)


def fp8_bmm_quant_triton(
    A: torch.Tensor,
    B: torch.Tensor,
    bias: torch.Tensor = None,
    *,
    quant_scale: torch.Tensor,
    out_dtype: torch.dtype = torch.float16,
    is_test=False,
):
    """``C[b] = (A[b] @ B[b]) * quant_scale + bias[b]`` cast to ``out_dtype``
    (fp8 outputs saturate).  A is [B,M,K], B is [B,K,N] (either major)."""
    del is_test
    Bs, M, K = A.shape
    N = B.shape[2]
    _lib.require_cuda(A, "A")
    C = torch.empty((Bs, M, N), dtype=out_dtype, device=A.device)
    if not torch.is_tensor(quant_scale):
        quant_scale = torch.tensor(float(quant_scale), device=A.device, dtype=torch.float32)
    scale = quant_scale if quant_scale.dtype == torch.float32 else quant_scale.float()
    return bmm_scaled(
        A, B, C,
        scale_a=scale.reshape(1), sa_strides=(0, 0, 0), qbm=1,
        scale_b=None, sb_strides=(0, 0, 0), qbn=1,
        qbk=max(K, 1), bias=bias, activation="none",
    )
