"""Per-block FP8 quantization and scaled BMM on sm_100a.

Drop-in for ``fp8_training/fp8_bench/impls/triton_per_block.py``: same
function signatures, validation and error messages, QuantResult layout and
registration scheme (``_register_block_scheme`` :436-537), with every launch
going to libpcb200 (pcb_quant_per_block, pcb_bmm_scaled).
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
    is_power_of_two,
    matrix_layout,
    resolve_operands,
)

_DEFAULT_QUANT_BLOCK_M = 128
_DEFAULT_QUANT_BLOCK_K = 128
_DEFAULT_QUANT_BLOCK_N = 128


def b200_per_block_quant(
    x: torch.Tensor,
    *,
    block_m: int = _DEFAULT_QUANT_BLOCK_M,
    block_n: int = _DEFAULT_QUANT_BLOCK_N,
    fp8_dtype: torch.dtype = torch.float8_e4m3fn,
    eps: float = 1e-12,
    profile: bool = False,
    pow2_scales: bool = False,
) -> QuantResult:
    """Per-block quantization (reference: triton_per_block_quant, :60-150).

    ``profile`` is accepted for signature compatibility; there is a single
    static kernel configuration.  ``pow2_scales`` selects the power-of-two
    (E8M0) scales of the FP8 training recipe (pcb_quant_per_block_pow2; not
    a reference option): every dequant scale is an exact power of two, which
    the block-scaled tensor-core GEMM applies in hardware.
    """
    del profile
    if x.ndim not in {2, 3}:
        raise ValueError(f"per-block quant expects a 2D or 3D tensor, got {tuple(x.shape)}")
    if not is_power_of_two(block_m) or not is_power_of_two(block_n):
        raise ValueError(
            "per-block quant currently requires power-of-two block sizes; "
            f"got block_m={block_m}, block_n={block_n}"
        )
    _lib.require_cuda(x, "x")
    output = torch.empty_like(x, dtype=fp8_dtype, memory_format=torch.preserve_format)
    if x.ndim == 2:
        batch = 1
        m, n = x.shape
        sxb = syb = 0
    else:
        batch, m, n = x.shape
        sxb, syb = x.stride(0), output.stride(0)
    m_blocks = (m + block_m - 1) // block_m
    n_blocks = (n + block_n - 1) // block_n
    scale_storage = torch.empty((batch, m_blocks, n_blocks), device=x.device, dtype=torch.float32)
    entry = "pcb_quant_per_block_pow2" if pow2_scales else "pcb_quant_per_block"
    _lib.check(
        getattr(_lib.lib(), entry)(
            x.data_ptr(), _lib.dtype_code(x.dtype), batch, m, n, sxb, x.stride(-2), x.stride(-1),
            output.data_ptr(), _lib.dtype_code(fp8_dtype), syb, output.stride(-2), output.stride(-1),
            scale_storage.data_ptr(), *scale_storage.stride(), block_m, block_n, eps,
            _lib.stream_ptr(x.device),
        ),
        entry,
    )
    dequant_scale = scale_storage.squeeze(0) if x.ndim == 2 else scale_storage
    return QuantResult(
        tensor=output,
        dequant_scale=dequant_scale,
        impl="b200_per_block",
        granularity="block",
        meta={
            "logical_shape": tuple(x.shape),
            "fp8_dtype": str(fp8_dtype),
            "block_m": block_m,
            "block_n": block_n,
            **({"scale_format": "e8m0"} if pow2_scales else {}),
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


def _validate_scale(value, *, expected_shape, expected_block_m, expected_block_n, operand) -> None:
    scale = value.dequant_scale
    if value.granularity != "block":
        raise ValueError(f"{operand} must use block granularity, got {value.granularity!r}")
    if tuple(scale.shape) != expected_shape:
        raise ValueError(f"{operand} dequant scale must have shape {expected_shape}, got {tuple(scale.shape)}")
    if scale.dtype != torch.float32:
        raise ValueError(f"{operand} dequant scale must be float32, got {scale.dtype}")
    if scale.device != value.tensor.device:
        raise ValueError(f"{operand} dequant scale must be on {value.tensor.device}, got {scale.device}")
    if value.meta.get("block_m") != expected_block_m or value.meta.get("block_n") != expected_block_n:
        raise ValueError(
            f"{operand} must be quantized with block_m={expected_block_m} "
            f"and block_n={expected_block_n}, "
            f"got block_m={value.meta.get('block_m')} "
            f"and block_n={value.meta.get('block_n')}"
        )


def _block_shape(value: QuantResult, operand: str) -> tuple[int, int]:
    if value.granularity != "block":
        raise ValueError(f"{operand} must use block granularity, got {value.granularity!r}")
    block_m = value.meta.get("block_m")
    block_n = value.meta.get("block_n")
    if not isinstance(block_m, int) or not isinstance(block_n, int) or block_m <= 0 or block_n <= 0:
        raise ValueError(f"{operand} has invalid per-block metadata: block_m={block_m}, block_n={block_n}")
    return block_m, block_n


def b200_per_block_bmm(
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
    """Per-block scaled BMM (reference: triton_per_block_bmm, :232-420).

    ``C[b] = act(sum_kg (A_kg @ B_kg) * (sa[b, m/QBM, kg] * sb[b, kg, n/QBN]) + bias)``.
    Operands are always fed by TMA; ``use_tma`` and ``profile`` are accepted
    for signature compatibility.
    """
    del profile, use_tma
    if a.tensor.ndim != 3 or b.tensor.ndim != 3:
        raise ValueError("BMM expects 3D quantized tensors")
    check_activation(activation)
    a_tensor, b_tensor = resolve_operands(a.tensor, b.tensor, do_transpose_a, do_transpose_b)
    batch, m, k = a_tensor.shape
    n = b_tensor.shape[-1]

    expected_block_m, expected_block_k = _block_shape(a, "A")
    b_block_k, expected_block_n = _block_shape(b, "B")
    if expected_block_k != b_block_k:
        raise ValueError(f"A and B must use the same K quant block: A={expected_block_k}, B={b_block_k}")
    if expected_block_k < 128 or expected_block_k % 128 != 0:
        raise ValueError(
            "the current per-block BMM configs require quant_block_k >= 128 "
            f"and divisible by 128, got {expected_block_k}"
        )
    num_blocks_m = (m + expected_block_m - 1) // expected_block_m
    num_blocks_k = (k + expected_block_k - 1) // expected_block_k
    num_blocks_n = (n + expected_block_n - 1) // expected_block_n
    _validate_scale(a, expected_shape=(batch, num_blocks_m, num_blocks_k), expected_block_m=expected_block_m,
                    expected_block_n=expected_block_k, operand="A")
    _validate_scale(b, expected_shape=(batch, num_blocks_k, num_blocks_n), expected_block_m=expected_block_k,
                    expected_block_n=expected_block_n, operand="B")
    out = check_out(out, batch, m, n, a_tensor.device, out_dtype)
    check_bias(bias, batch, m, n, a_tensor.device, require_n_contiguous=True)
    sa, sb = a.dequant_scale, b.dequant_scale
    # Both operands with power-of-two (E8M0) scales and 128-deep K blocks: the
    # tensor core applies the scales (pcb_bmm_block_scaled).
    block_scaled = (a.meta.get("scale_format") == "e8m0" and b.meta.get("scale_format") == "e8m0"
                    and expected_block_k == 128)
    return bmm_scaled(
        a_tensor, b_tensor, out,
        scale_a=sa, sa_strides=(sa.stride(0), sa.stride(1), sa.stride(2)), qbm=expected_block_m,
        scale_b=sb, sb_strides=(sb.stride(0), sb.stride(1), sb.stride(2)), qbn=expected_block_n,
        qbk=expected_block_k, bias=bias, activation=activation, block_scaled=block_scaled,
    )


def _register_block_scheme(quant_impl, *, a_block, b_block, description, register_quant_impl=True,
                           pow2_scales=False):
    """Register one quant impl plus its five BMM layouts (reference :436-521)."""
    quant_a_kwargs = {"block_m": a_block[0], "block_n": a_block[1]}
    quant_b_kwargs = {"block_m": b_block[0], "block_n": b_block[1]}
    if pow2_scales:
        quant_a_kwargs["pow2_scales"] = quant_b_kwargs["pow2_scales"] = True
    if register_quant_impl:
        register_quant(
            quant_impl,
            partial(b200_per_block_quant, block_m=a_block[0], block_n=a_block[1], pow2_scales=pow2_scales),
            description,
        )
    common = {"quant_impl": quant_impl, "quant_a_kwargs": quant_a_kwargs, "quant_b_kwargs": quant_b_kwargs}
    register_bmm(
        f"{quant_impl}_a_k_b_n",
        partial(b200_per_block_bmm, do_transpose_b=False),
        layout="n",
        prepare_b=lambda value: prepare_b_layout(value, "n"),
        description="Per-block FP8 BMM with an N-major [B,K,N] right operand (MN-major UMMA descriptor).",
        **common,
    )
    register_bmm(
        f"{quant_impl}_a_k_b_k",
        partial(b200_per_block_bmm, do_transpose_b=False),
        layout="k",
        prepare_b=lambda value: prepare_b_layout(value, "k"),
        description="Per-block FP8 BMM with a prepacked K-major right operand.",
        **common,
    )
    register_bmm(
        f"{quant_impl}_a_k_b_n_transpose",
        partial(b200_per_block_bmm, do_transpose_b=True),
        layout="n",
        prepare_b=lambda value: prepare_b_layout(value, "n"),
        description="N-major per-block FP8 BMM with packing inside the call.",
        **common,
    )
    register_bmm(
        f"{quant_impl}_a_m_b_n",
        partial(b200_per_block_bmm, do_transpose_a=False, do_transpose_b=False),
        a_layout="m",
        layout="n",
        prepare_a=lambda value: prepare_a_layout(value, "m"),
        prepare_b=lambda value: prepare_b_layout(value, "n"),
        description="Per-block FP8 BMM with direct M-major A and N-major B operands.",
        **common,
    )
    register_bmm(
        f"{quant_impl}_a_m_transpose_b_n_transpose",
        partial(b200_per_block_bmm, do_transpose_a=True, do_transpose_b=True),
        a_layout="m",
        layout="n",
        prepare_a=lambda value: prepare_a_layout(value, "m"),
        prepare_b=lambda value: prepare_b_layout(value, "n"),
        description="M-major A and N-major B packed inside the per-block BMM call.",
        **common,
    )


def register_all(prefix: str) -> None:
    _register_block_scheme(f"{prefix}_per_block_1d", a_block=(1, _DEFAULT_QUANT_BLOCK_K),
                           b_block=(_DEFAULT_QUANT_BLOCK_K, 1),
                           description="1D K-block scale quantization; defaults to 1x128 blocks.")
    _register_block_scheme(f"{prefix}_per_block_2d", a_block=(_DEFAULT_QUANT_BLOCK_M, _DEFAULT_QUANT_BLOCK_K),
                           b_block=(_DEFAULT_QUANT_BLOCK_K, _DEFAULT_QUANT_BLOCK_N),
                           description="2D block scale quantization; defaults to 128x128 blocks.")
