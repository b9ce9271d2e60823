"""CPU restatement of the reference's FP8 quantizers (TEST INFRASTRUCTURE ONLY).

Every function evaluates the reference's own expressions with eager torch on
the CPU, so the float semantics are the ones torch gives them:

* ``fp8_max / amax`` (python scalar / tensor) is evaluated by torch as
  ``amax.reciprocal() * fp8_max`` -- two roundings, NOT one IEEE divide.
* ``1.0 / quant_scale`` and ``quant_scale.reciprocal()`` are one IEEE
  reciprocal.
* ``amax / fp8_max`` (tensor / python scalar) is one IEEE divide on the CPU.
* ``clamp`` runs before the fp8 cast, so the cast never overflows
  (torch's CPU cast would turn an overflow into NaN).
* ``amax`` propagates NaN; ``clamp_min(eps)`` keeps a NaN.

The CUDA kernels reproduce exactly these operations (``__frcp_rn`` then
``__fmul_rn`` for the quant scale, ``__fdiv_rn`` for the per-channel dequant
scale, ``cvt.rn.satfinite`` for the cast), which is what makes the
bit-exact parity tests possible.
"""

from __future__ import annotations

import torch

FP8_MAX = {
    torch.float8_e4m3fn: 448.0,
    torch.float8_e5m2: 57344.0,
}


def _fp8_max(fp8_dtype: torch.dtype) -> float:
    return float(torch.finfo(fp8_dtype).max)


def per_block_quant(
    x: torch.Tensor,
    *,
    block_m: int = 128,
    block_n: int = 128,
    fp8_dtype: torch.dtype = torch.float8_e4m3fn,
    eps: float = 1e-12,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-block quantization.

    Follows ``fp8_training/fp8_bench/kernels/quant/per_block.py:35-48``
    (amax over one ``block_m x block_n`` tile, masked tails read as 0,
    ``quant_scale = fp8_max / max(amax, eps)``, ``dequant = 1.0 / quant_scale``,
    ``y = clamp(x * quant_scale)``) and the scale storage of
    ``impls/triton_per_block.py:79-100,138`` (``[B, m_blocks, n_blocks]``,
    squeezed to 2D for a 2D input).
    """
    if x.ndim not in (2, 3):
        raise ValueError(f"per-block quant expects a 2D or 3D tensor, got {tuple(x.shape)}")
    squeeze = x.ndim == 2
    xb = x.unsqueeze(0) if squeeze else x
    batch, m, n = xb.shape
    mb = (m + block_m - 1) // block_m
    nb = (n + block_n - 1) // block_n
    xf = torch.zeros((batch, mb * block_m, nb * block_n), dtype=torch.float32)
    xf[:, :m, :n] = xb.float()
    tiles = xf.view(batch, mb, block_m, nb, block_n)
    x_amax = tiles.abs().amax(dim=(2, 4))
    x_safe_amax = x_amax.clamp_min(eps)
    fp8_max = _fp8_max(fp8_dtype)
    quant_scale = fp8_max / x_safe_amax
    dequant_scale = 1.0 / quant_scale
    qs_full = quant_scale.repeat_interleave(block_m, dim=1).repeat_interleave(block_n, dim=2)
    y = torch.clamp(xf * qs_full, min=-fp8_max, max=fp8_max)[:, :m, :n].to(fp8_dtype)
    if squeeze:
        return y[0], dequant_scale[0]
    return y, dequant_scale


def per_block_quant_pow2(
    x: torch.Tensor,
    *,
    block_m: int = 128,
    block_n: int = 128,
    fp8_dtype: torch.dtype = torch.float8_e4m3fn,
    eps: float = 1e-12,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-block quantization with power-of-two (E8M0) scales.

    Restates ``pcb_quant_per_block_pow2`` (the FP8 training recipe of this
    library; the reference has no counterpart): ``r = RN(max(amax, eps) /
    fp8_max)`` in fp32, ``e`` the smallest integer with ``2**e >= r`` (from
    r's exponent and mantissa bits), ``quant_scale = 2**-e``, ``dequant =
    1 / quant_scale``; a zero or subnormal ``r`` is clamped to ``2**-126``
    (``quant_scale = 2**126``) and a non-finite ``r`` gives ``quant_scale =
    1 / r``.  Tiles, tails and storage as :func:`per_block_quant`.
    """
    if x.ndim not in (2, 3):
        raise ValueError(f"per-block quant expects a 2D or 3D tensor, got {tuple(x.shape)}")
    squeeze = x.ndim == 2
    xb = x.unsqueeze(0) if squeeze else x
    batch, m, n = xb.shape
    mb = (m + block_m - 1) // block_m
    nb = (n + block_n - 1) // block_n
    xf = torch.zeros((batch, mb * block_m, nb * block_n), dtype=torch.float32)
    xf[:, :m, :n] = xb.float()
    tiles = xf.view(batch, mb, block_m, nb, block_n)
    safe = tiles.abs().amax(dim=(2, 4)).clamp_min(eps)
    fp8_max = _fp8_max(fp8_dtype)
    r = safe / fp8_max
    bits = r.view(torch.int32)
    ef = (bits >> 23) & 0xFF
    e = ef - 127 + ((bits & 0x7FFFFF) != 0).to(torch.int32)
    pow2 = ((127 - e).clamp(0, 254) << 23).view(torch.float32)
    pow2 = torch.where(ef == 0, torch.tensor(2.0 ** 126, dtype=torch.float32), pow2)
    quant_scale = torch.where(ef == 0xFF, 1.0 / r, pow2)
    dequant_scale = 1.0 / quant_scale
    qs_full = quant_scale.repeat_interleave(block_m, dim=1).repeat_interleave(block_n, dim=2)
    y = torch.clamp(xf * qs_full, min=-fp8_max, max=fp8_max)[:, :m, :n].to(fp8_dtype)
    if squeeze:
        return y[0], dequant_scale[0]
    return y, dequant_scale


def per_channel_quant(
    x: torch.Tensor,
    *,
    channel_axis: int = -1,
    fp8_dtype: torch.dtype = torch.float8_e4m3fn,
    eps: float = 1e-12,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-channel quantization.

    The eager body of ``fp8_per_channel_quant_torch_compile``
    (``fp8_training/fp8_bench/kernels/quant/per_channel.py:9-29``):
    ``channel_axis=-2`` keeps one scale per row (reduce over the last dim),
    ``-1`` one scale per column (reduce over rows); ``dequant = amax / fp8_max``.
    """
    if channel_axis not in (-1, -2):
        raise ValueError(f"channel_axis must be -1 or -2, got {channel_axis}")
    reduction_dim = -1 if channel_axis == -2 else -2
    x_safe_amax = torch.amax(torch.abs(x.float()), dim=reduction_dim).clamp_min(eps)
    fp8_max = _fp8_max(fp8_dtype)
    quant_scale = fp8_max / x_safe_amax
    dequant_scale = x_safe_amax / fp8_max
    output = torch.clamp(
        x.float() * quant_scale.unsqueeze(reduction_dim),
        min=-fp8_max,
        max=fp8_max,
    ).to(fp8_dtype)
    return output, dequant_scale


def per_tensor_quant(
    x: torch.Tensor,
    *,
    fp8_dtype: torch.dtype = torch.float8_e4m3fn,
    eps: float = 1e-12,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-tensor quantization of ``impls/triton_per_tensor.py:41-44`` plus the
    cast kernel ``kernels/quant/per_tensor.py:37-43``.

    Returns ``(y, dequant_scale)`` with a 0-dim fp32 dequant scale.
    """
    x_min, x_max = x.aminmax()
    max_abs = torch.maximum(x_min.abs(), x_max.abs()).float().clamp(min=eps)
    fp8_max = _fp8_max(fp8_dtype)
    quant_scale = fp8_max / max_abs
    dequant_scale = quant_scale.reciprocal()
    y = torch.clamp(x.float() * quant_scale, min=-fp8_max, max=fp8_max).to(fp8_dtype)
    return y, dequant_scale


def legacy_per_tensor_quant(
    x: torch.Tensor,
    quant_dtype: torch.dtype = torch.float8_e4m3fn,
    fp8_range: float = 448.0,
    eps: float = 1e-12,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Legacy ``fp8_quant_triton`` (``kernels/fp8_bmm/fp8_warper.py:19-25``) with
    the clamp of its cast kernel (``kernel/fp8_quant_kernel.py:57-58``).

    Unlike the fp8_bench path, the scale arithmetic stays in ``x``'s dtype
    (no ``.float()``), so a bf16 input gets a bf16 quant scale.
    """
    x_min, x_max = x.aminmax()
    x_max_abs = torch.maximum(x_min.abs(), x_max.abs())
    x_max_abs = x_max_abs.clamp(min=eps)
    quant_factor = fp8_range / x_max_abs
    reciprocal_factor = quant_factor.reciprocal()
    y = torch.clamp(
        x.float() * quant_factor.float(), min=-fp8_range, max=fp8_range
    ).to(quant_dtype)
    return y, reciprocal_factor


def float8_dynamic_cast(
    x: torch.Tensor,
    fp8_dtype: torch.dtype = torch.float8_e4m3fn,
    *,
    axiswise: bool = False,
    eps: float = 1e-12,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Dynamic float8 cast of the FP8 training linear.

    ``hp_tensor_to_float8_dynamic``
    (``fp8_training/fp8_bench/modules/float8/float8_scaling_utils.py:29-72``):
    amax over the whole tensor, or per row over the last dim when
    ``axiswise`` (``tensor_to_amax``, ``float8_utils.py:56-86``, keepdim);
    ``scale = f32(fp8_max / clamp(f64(amax), eps))`` (``amax_to_scale``,
    ``:31-53``); ``data = fp8(clamp(f32(x) * scale, +-fp8_max))``
    (``to_fp8_saturated`` ``:118-139``, ``float8_training_tensor.py:150-155``).
    Returns ``(data, scale)``; the scale is the QUANT scale.
    """
    xf = x.float()
    amax = xf.abs().amax(dim=-1, keepdim=True) if axiswise else xf.abs().max()
    fmax = torch.finfo(fp8_dtype).max
    scale = (fmax / torch.clamp(amax.to(torch.float64), min=eps)).to(torch.float32)
    data = torch.clamp(xf * scale, min=-fmax, max=fmax).to(fp8_dtype)
    return data, scale


def dequantize(
    tensor: torch.Tensor,
    dequant_scale: torch.Tensor,
    granularity: str,
    meta: dict,
    dtype: torch.dtype = torch.float32,
) -> torch.Tensor:
    """``QuantResult.dequantize`` (``fp8_training/fp8_bench/registry.py:18-70``)."""
    scale = dequant_scale.to(dtype)
    if granularity == "tensor":
        return tensor.to(dtype) * scale
    if granularity == "channel":
        axis = meta["channel_axis"]
        scale = scale.unsqueeze(-1 if axis == -2 else -2)
        return tensor.to(dtype) * scale
    if granularity == "block":
        bm, bn = meta["block_m"], meta["block_n"]
        m, n = tensor.shape[-2:]
        rows = torch.arange(m) // bm
        cols = torch.arange(n) // bn
        scale = scale.index_select(-2, rows).index_select(-1, cols)
        return tensor.to(dtype).mul_(scale)
    raise ValueError(f"unknown quantization granularity: {granularity}")
