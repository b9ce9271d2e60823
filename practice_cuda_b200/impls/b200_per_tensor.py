"""Per-tensor FP8 quantization and scaled BMM on sm_100a.

Drop-in for ``fp8_training/fp8_bench/impls/triton_per_tensor.py`` (quant
:28-96, BMM :140-305).  The amax, the scale arithmetic and the cast all run in
libpcb200 (two launches; no host synchronisation).
"""

from __future__ import annotations

from functools import partial
from typing import Optional

import torch

from .. import _lib
from ..registry import QuantResult, register_bmm, register_quant
from ._common import (
    a_layout,
    bmm_scaled,
    check_activation,
    check_bias,
    check_out,
    matrix_layout,
    resolve_operands,
)


def quantize_per_tensor(x: torch.Tensor, fp8_dtype: torch.dtype, fp8_max: float, eps: float,
                        scale_dtype: torch.dtype = torch.float32):
    """Returns (fp8 tensor, quant_scale, dequant_scale); scales are 0-dim fp32
    tensors whose values are exact in ``scale_dtype``."""
    _lib.require_cuda(x, "x")
    output = torch.empty_like(x, dtype=fp8_dtype, memory_format=torch.preserve_format)
    if x.ndim == 2:
        batch = 1
        m, n = x.shape
        sxb = syb = 0
    elif x.ndim == 3:
        batch, m, n = x.shape
        sxb, syb = x.stride(0), output.stride(0)
    else:
        raise ValueError(f"per-tensor quant expects a 2D or 3D tensor, got shape={tuple(x.shape)}")
    lib = _lib.lib()
    scales = torch.empty(2, device=x.device, dtype=torch.float32)
    workspace = torch.empty(lib.pcb_quant_per_tensor_workspace_floats(), device=x.device, dtype=torch.float32)
    _lib.check(
        lib.pcb_quant_per_tensor(
            x.data_ptr(), _lib.dtype_code(x.dtype), batch, m, n, sxb, x.stride(-2), x.stride(-1),
            output.data_ptr(), _lib.dtype_code(fp8_dtype), syb, output.stride(-2), output.stride(-1),
            scales[0:1].data_ptr(), scales[1:2].data_ptr(), _lib.dtype_code(scale_dtype), fp8_max, eps,
            workspace.data_ptr(), _lib.stream_ptr(x.device),
        ),
        "pcb_quant_per_tensor",
    )
    return output, scales[0], scales[1]


def b200_per_tensor_quant(
    x: torch.Tensor,
    *,
    fp8_dtype: torch.dtype = torch.float8_e4m3fn,
    eps: float = 1e-12,
    profile: bool = False,
) -> QuantResult:
    """Per-tensor quantization (reference: triton_per_tensor_quant, :28-96)."""
    del profile
    if x.ndim not in {2, 3}:
        raise ValueError(f"per-tensor quant expects a 2D or 3D tensor, got shape={tuple(x.shape)}")
    output, _, dequant_scale = quantize_per_tensor(x, fp8_dtype, float(torch.finfo(fp8_dtype).max), eps)
    return QuantResult(
        tensor=output,
        dequant_scale=dequant_scale,
        impl="b200_per_tensor",
        granularity="tensor",
        meta={"logical_shape": tuple(x.shape), "fp8_dtype": str(fp8_dtype)},
    )


def prepare_a_layout(value: QuantResult, layout: str) -> QuantResult:
    if layout not in {"k", "m"}:
        raise ValueError(f"unknown A layout: {layout}")
    actual = a_layout(value.tensor)
    expected = f"{layout}-major"
    if actual != expected:
        raise ValueError(f"expected {expected} A, got {actual}")
    return value


def prepare_b_layout(value: QuantResult, layout: str) -> QuantResult:
    if layout not in {"n", "k"}:
        raise ValueError(f"unknown B layout: {layout}")
    actual = matrix_layout(value.tensor, "B")
    expected = f"{layout}-major"
    if actual != expected:
        raise ValueError(f"expected {expected} B, got {actual}")
    return value


def b200_per_tensor_bmm(
    a: QuantResult,
    b: QuantResult,
    *,
    out_dtype: torch.dtype = torch.bfloat16,
    bias: Optional[torch.Tensor] = None,
    out: Optional[torch.Tensor] = None,
    do_transpose_a: bool = False,
    do_transpose_b: bool = False,
    dequant_scale: Optional[torch.Tensor] = None,
    profile: bool = False,
    use_tma: bool = False,
    activation: str = "none",
) -> torch.Tensor:
    """Per-tensor scaled BMM (reference: triton_per_tensor_bmm, :140-305):
    ``C = act((A @ B) * s + bias)`` with ``s = a.scale * b.scale`` (formed in
    fp32 on the device) unless ``dequant_scale`` is given."""
    del profile, use_tma
    if a.tensor.ndim != 3 or b.tensor.ndim != 3:
        raise ValueError("BMM expects 3D quantized tensors")
    check_activation(activation)
    a_tensor, b_tensor = resolve_operands(a.tensor, b.tensor, do_transpose_a, do_transpose_b)
    batch, m, k = a_tensor.shape
    n = b_tensor.shape[-1]
    out = check_out(out, batch, m, n, a_tensor.device, out_dtype)
    check_bias(bias, batch, m, n, a_tensor.device, require_n_contiguous=False)
    if dequant_scale is not None:
        sa, sb = dequant_scale, None
    else:
        sa, sb = a.dequant_scale, b.dequant_scale
    for s in (sa, sb):
        if s is None:
            continue
        if s.numel() != 1:
            raise ValueError(f"per-tensor BMM expects one combined dequant scale, got shape={tuple(s.shape)}")
        if s.dtype != torch.float32:
            raise ValueError(f"dequant_scale must be float32, got {s.dtype}")
        if s.device != a_tensor.device:
            raise ValueError(
                f"dequant_scale must be on the same device as A and B: scale={s.device}, tensors={a_tensor.device}"
            )
    return bmm_scaled(
        a_tensor, b_tensor, out,
        scale_a=sa, sa_strides=(0, 0, 0), qbm=1,
        scale_b=sb, sb_strides=(0, 0, 0), qbn=1,
        qbk=max(k, 1), bias=bias, activation=activation,
    )


def register_all(prefix: str) -> None:
    quant = f"{prefix}_per_tensor"
    register_quant(quant, b200_per_tensor_quant, "Per-tensor scale quantization; supports E4M3 and E5M2.")
    common = {"quant_impl": quant}
    register_bmm(f"{quant}_a_k_b_n", partial(b200_per_tensor_bmm, do_transpose_b=False), layout="n",
                 prepare_b=lambda v: prepare_b_layout(v, "n"),
                 description="Per-tensor FP8 BMM with an N-major [B,K,N] right operand.", **common)
    register_bmm(f"{quant}_a_k_b_k", partial(b200_per_tensor_bmm, do_transpose_b=False), layout="k",
                 prepare_b=lambda v: prepare_b_layout(v, "k"),
                 description="Per-tensor FP8 BMM with a prepacked K-major right operand.", **common)
    register_bmm(f"{quant}_a_k_b_n_transpose", partial(b200_per_tensor_bmm, do_transpose_b=True), layout="n",
                 prepare_b=lambda v: prepare_b_layout(v, "n"),
                 description="N-major per-tensor FP8 BMM with packing inside the call.", **common)
    register_bmm(f"{quant}_a_m_b_n", partial(b200_per_tensor_bmm, do_transpose_a=False, do_transpose_b=False),
                 a_layout="m", layout="n", prepare_a=lambda v: prepare_a_layout(v, "m"),
                 prepare_b=lambda v: prepare_b_layout(v, "n"),
                 description="Per-tensor FP8 BMM with direct M-major A and N-major B operands.", **common)
    register_bmm(f"{quant}_a_m_transpose_b_n_transpose",
                 partial(b200_per_tensor_bmm, do_transpose_a=True, do_transpose_b=True),
                 a_layout="m", layout="n", prepare_a=lambda v: prepare_a_layout(v, "m"),
                 prepare_b=lambda v: prepare_b_layout(v, "n"),
                 description="M-major A and N-major B packed inside the per-tensor BMM call.", **common)
