"""Per-channel FP8 quantization and scaled BMM on sm_100a.

Drop-in for ``fp8_training/fp8_bench/impls/triton_per_channel.py`` (quant
:90-219, BMM :271-427, registrations :443-525) and for the torch quantizer
``fp8_per_channel_quant_torch_compile`` (``kernels/quant/per_channel.py:9-29``),
whose numerics the kernel reproduces bit for bit.
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


def quantize_per_channel(x: torch.Tensor, channel_axis: int, fp8_dtype: torch.dtype, eps: float):
    """(fp8 tensor, fp32 dequant scale) -- the torch quantizer's return shape."""
    if x.ndim not in {2, 3}:
        raise ValueError(f"per-channel quant expects a 2D or 3D tensor, got {tuple(x.shape)}")
    if channel_axis not in {-1, -2}:
        raise ValueError(f"channel_axis must be -1 or -2, got {channel_axis}")
    _lib.require_cuda(x, "x")
    output = torch.empty_like(x, dtype=fp8_dtype, memory_format=torch.preserve_format)
    if x.ndim == 2:
        batch = 1
        m, n = x.shape
        sxb = syb = 0
    else:
        batch, m, n = x.shape
        sxb, syb = x.stride(0), output.stride(0)
    channels = m if channel_axis == -2 else n
    scale_storage = torch.empty((batch, channels), device=x.device, dtype=torch.float32)
    _lib.check(
        _lib.lib().pcb_quant_per_channel(
            x.data_ptr(), _lib.dtype_code(x.dtype), batch, m, n, sxb, x.stride(-2), x.stride(-1),
            output.data_ptr(), _lib.dtype_code(fp8_dtype), syb, output.stride(-2), output.stride(-1),
            scale_storage.data_ptr(), scale_storage.stride(0), scale_storage.stride(1),
            channel_axis, eps, _lib.stream_ptr(x.device),
        ),
        "pcb_quant_per_channel",
    )
    return output, (scale_storage.squeeze(0) if x.ndim == 2 else scale_storage)


def b200_per_channel_quant(
    x: torch.Tensor,
    *,
    channel_axis: int = -1,
    fp8_dtype: torch.dtype = torch.float8_e4m3fn,
    eps: float = 1e-12,
    profile: bool = False,
    one_pass: bool = False,
) -> QuantResult:
    """Per-channel quantization (reference: triton_per_channel_quant, :90-219).

    ``one_pass`` keeps the reference's argument checks (reduction <= 4096);
    the kernel choice does not depend on it.
    """
    del profile
    if x.ndim not in {2, 3}:
        raise ValueError(f"per-channel quant expects a 2D or 3D tensor, got {tuple(x.shape)}")
    if channel_axis not in {-1, -2}:
        raise ValueError(f"channel_axis must be -1 or -2, got {channel_axis}")
    matrix_layout(x, "quant input")
    if one_pass:
        m, n = x.shape[-2:]
        reduction_size = n if channel_axis == -2 else m
        if reduction_size == 0:
            raise ValueError("one-pass per-channel quant requires a non-empty reduction")
        if reduction_size > 4096:
            raise ValueError(
                f"one-pass per-channel quant supports reduction sizes up to 4096, got {reduction_size}"
            )
    output, dequant_scale = quantize_per_channel(x, channel_axis, fp8_dtype, eps)
    return QuantResult(
        tensor=output,
        dequant_scale=dequant_scale,
        impl="b200_per_channel",
        granularity="channel",
        meta={
            "logical_shape": tuple(x.shape),
            "fp8_dtype": str(fp8_dtype),
            "channel_axis": channel_axis,
            "quant_strategy": "one_pass" if one_pass else "b200",
        },
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


def _validate_scale(value, *, expected_shape, expected_axis, operand) -> None:
    scale = value.dequant_scale
    if scale.shape != expected_shape:
        raise ValueError(f"{operand} dequant scale must have shape {expected_shape}, got {tuple(scale.shape)}")
    if scale.dtype != torch.float32:
        raise ValueError(f"{operand} dequant scale must be float32, got {scale.dtype}")
    if scale.device != value.tensor.device:
        raise ValueError(f"{operand} dequant scale must be on {value.tensor.device}, got {scale.device}")
    if value.meta.get("channel_axis") != expected_axis:
        raise ValueError(
            f"{operand} must be quantized with channel_axis={expected_axis}, got {value.meta.get('channel_axis')}"
        )


def b200_per_channel_bmm(
    a: QuantResult,
    b: QuantResult,
    *,
    out_dtype: torch.dtype = torch.bfloat16,
    bias: Optional[torch.Tensor] = None,
    out: Optional[torch.Tensor] = None,
    do_transpose_a: bool = False,
    do_transpose_b: bool = False,
    profile: bool = False,
    use_tma: bool = False,
    activation: str = "none",
) -> torch.Tensor:
    """Per-channel scaled BMM (reference: triton_per_channel_bmm, :271-427):
    ``C = act((A @ B) * sa[m] * sb[n] + bias)``, scales in the epilogue."""
    del profile, use_tma
    if a.tensor.ndim != 3 or b.tensor.ndim != 3:
        raise ValueError("BMM expects 3D quantized tensors")
    check_activation(activation)
    a_tensor, b_tensor = resolve_operands(a.tensor, b.tensor, do_transpose_a, do_transpose_b)
    batch, m, k = a_tensor.shape
    n = b_tensor.shape[-1]
    _validate_scale(a, expected_shape=(batch, m), expected_axis=-2, operand="A")
    _validate_scale(b, expected_shape=(batch, n), expected_axis=-1, operand="B")
    out = check_out(out, batch, m, n, a_tensor.device, out_dtype)
    check_bias(bias, batch, m, n, a_tensor.device, require_n_contiguous=False)
    sa, sb = a.dequant_scale, b.dequant_scale
    return bmm_scaled(
        a_tensor, b_tensor, out,
        scale_a=sa, sa_strides=(sa.stride(0), sa.stride(1), 0), qbm=1,
        scale_b=sb, sb_strides=(sb.stride(0), 0, sb.stride(1)), qbn=1,
        qbk=max(k, 1), bias=bias, activation=activation,
    )


def per_channel_quant_torch_compile(x, channel_axis, fp8_dtype, eps):
    """Signature of ``microbench/profile_fused_quant.py:3-23`` and
    ``kernels/quant/per_channel.py:9-29``: returns ``(output, dequant_scale)``."""
    return quantize_per_channel(x, channel_axis, fp8_dtype, eps)


def register_all(prefix: str) -> None:
    quant = f"{prefix}_per_channel"
    register_quant(quant, b200_per_channel_quant, "Per-channel scale quantization; supports E4M3 and E5M2.")
    register_quant(f"{quant}_one_pass", partial(b200_per_channel_quant, one_pass=True),
                   "Per-channel quantization with the one-pass argument limits (reduction <= 4096).")
    if prefix == "triton":
        register_quant("torch_compile_per_channel", b200_per_channel_quant,
                       "Per-channel quantization (stands in for the torch.compile quantizer).")
    common = {"quant_impl": quant, "quant_a_kwargs": {"channel_axis": -2}, "quant_b_kwargs": {"channel_axis": -1}}
    register_bmm(f"{quant}_a_k_b_n", partial(b200_per_channel_bmm, do_transpose_b=False), layout="n",
                 prepare_b=lambda v: prepare_b_layout(v, "n"),
                 description="Per-channel FP8 BMM with an N-major [B,K,N] right operand.", **common)
    register_bmm(f"{quant}_a_k_b_k", partial(b200_per_channel_bmm, do_transpose_b=False), layout="k",
                 prepare_b=lambda v: prepare_b_layout(v, "k"),
                 description="Per-channel FP8 BMM with a prepacked K-major right operand.", **common)
    register_bmm(f"{quant}_a_k_b_n_transpose", partial(b200_per_channel_bmm, do_transpose_b=True), layout="n",
                 prepare_b=lambda v: prepare_b_layout(v, "n"),
                 description="N-major per-channel FP8 BMM with packing inside the call.", **common)
    register_bmm(f"{quant}_a_m_b_n", partial(b200_per_channel_bmm, do_transpose_a=False, do_transpose_b=False),
                 a_layout="m", layout="n", prepare_a=lambda v: prepare_a_layout(v, "m"),
                 prepare_b=lambda v: prepare_b_layout(v, "n"),
                 description="Per-channel FP8 BMM with direct M-major A and N-major B operands.", **common)
    register_bmm(f"{quant}_a_m_transpose_b_n_transpose",
                 partial(b200_per_channel_bmm, do_transpose_a=True, do_transpose_b=True),
                 a_layout="m", layout="n", prepare_a=lambda v: prepare_a_layout(v, "m"),
                 prepare_b=lambda v: prepare_b_layout(v, "n"),
                 description="M-major A and N-major B with both operands packed inside the BMM call.", **common)
