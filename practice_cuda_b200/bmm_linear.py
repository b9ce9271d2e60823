"""Batched FP8 training linear on libpcb200 (drop-in for the reference's
``Float8BMMLinear``).

The reference module (``fp8_training/fp8_bench/modules/bmm_linear.py``)
trains a batched dense layer -- weight ``[B, N, K]``, bias ``[B, N]``, input
``[B, M, K]`` -- with dynamic FP8 casts (tensorwise or axiswise scales,
E4M3 input and weight, E5M2 gradient) and three scaled FP8 BMMs per step,
all through the Triton op ``fp8_bench::bmm_linear_tma`` (``:121-227``).  Here

* :func:`bmm_linear_tma` is the same op (``pcb200::bmm_linear_tma``, same
  arguments and semantics: ``(A @ B) / (scale_a * scale_b) + bias`` with the
  QUANT scales of the casts) on ``pcb_bmm_scaled`` / ``pcb_bmm_scaled_mixed``;
* the casts run on ``pcb_quant_float8_dynamic`` with the reference's
  numerics (``scale = fp8_max / max(amax, eps)``, saturating cast;
  ``float8_utils.py:31-53, 118-139``);
* :class:`Float8BMMLinear`, :class:`BMMLinear`,
  :func:`convert_to_float8_bmm_training` keep the reference's constructor
  arguments, shapes and errors, and the backward's scale folding for
  axiswise scaling (``bmm_linear.py:375-451``).

FP8 all-gather of this module's weights under FSDP2 is not provided (the
per-block all-gather lives in :mod:`practice_cuda_b200.fsdp_fp8`).
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn as nn

from . import _lib
from .impls._common import bmm_scaled

E4M3 = torch.float8_e4m3fn
E5M2 = torch.float8_e5m2
EPS = 1e-12  # float8_utils.EPS


# --------------------------------------------------------------------- config ---
@dataclass(frozen=True)
class Float8BMMLinearConfig:
    """The parts of the reference's ``Float8BMMLinearConfig``
    (``bmm_linear.py:40-85``) this module reads: one scaling granularity for
    all six casts (dynamic only), E4M3 input/weight and E5M2 grad-output.
    A reference/torchAO config object is accepted too (see :func:`_resolve`)."""

    scaling_granularity: str = "tensorwise"  # or "axiswise"
    input_dtype: torch.dtype = E4M3
    weight_dtype: torch.dtype = E4M3
    grad_output_dtype: torch.dtype = E5M2
    enable_fsdp_float8_all_gather: bool = False

    def __post_init__(self) -> None:
        if self.scaling_granularity not in ("tensorwise", "axiswise"):
            raise ValueError("Float8BMMLinear's TMA backend does not support scaling "
                             f"{self.scaling_granularity!r}")
        for d in (self.input_dtype, self.weight_dtype, self.grad_output_dtype):
            if d not in (E4M3, E5M2):
                raise ValueError(f"unsupported float8 dtype {d}")
        if self.enable_fsdp_float8_all_gather:
            raise ValueError("FP8 all-gather of Float8BMMLinear weights is not supported by this backend")


def _resolve(config) -> Float8BMMLinearConfig:
    """Map a reference / torchAO ``Float8LinearConfig`` (``cast_config_*``
    with ``scaling_granularity`` / ``target_dtype``) onto this config."""
    if config is None:
        return Float8BMMLinearConfig()
    if isinstance(config, Float8BMMLinearConfig):
        return config
    gran = getattr(config.cast_config_input.scaling_granularity, "name", str(config.cast_config_input.scaling_granularity))
    return Float8BMMLinearConfig(
        scaling_granularity=gran.lower(),
        input_dtype=config.cast_config_input.target_dtype,
        weight_dtype=config.cast_config_weight.target_dtype,
        grad_output_dtype=config.cast_config_grad_output.target_dtype,
        enable_fsdp_float8_all_gather=bool(getattr(config, "enable_fsdp_float8_all_gather", False)),
    )


# ---------------------------------------------------------------------- casts ---
def cast_to_float8(x: torch.Tensor, dtype: torch.dtype, axiswise: bool) -> tuple[torch.Tensor, torch.Tensor]:
    """Dynamic FP8 cast of a [B, M, K] (or [M, K]) tensor: ``(data, scale)``
    with ``scale = fp8_max / max(amax, 1e-12)`` per tensor (a 0-dim scale) or
    per row over the last dim (``axiswise``: scale [B, M, 1]), ``data =
    sat(fp8(x * scale))`` -- ``hp_tensor_to_float8_dynamic``
    (``float8_scaling_utils.py:29-72``) with ``axiswise_dim=-1``."""
    _lib.require_cuda(x, "x")
    squeeze = x.ndim == 2
    x3 = x.unsqueeze(0) if squeeze else x
    if x3.ndim != 3:
        raise ValueError(f"expected a 2D or 3D tensor, got {tuple(x.shape)}")
    if x3.dtype not in (torch.float32, torch.float16, torch.bfloat16):
        x3 = x3.float()
    batch, m, n = x3.shape
    data = torch.empty((batch, m, n), device=x.device, dtype=dtype)
    lib = _lib.lib()
    if axiswise:
        scale = torch.empty((batch, m, 1), device=x.device, dtype=torch.float32)
        ws = None
        ss = (scale.stride(0), scale.stride(1))
    else:
        scale = torch.empty((), device=x.device, dtype=torch.float32)
        ws = torch.empty((lib.pcb_quant_per_tensor_workspace_floats(),), device=x.device, dtype=torch.float32)
        ss = (0, 0)
    _lib.check(
        lib.pcb_quant_float8_dynamic(
            x3.data_ptr(), _lib.dtype_code(x3.dtype), batch, m, n, *x3.stride(),
            data.data_ptr(), _lib.dtype_code(dtype), *data.stride(),
            scale.data_ptr(), *ss, 1 if axiswise else 0, EPS,
            ws.data_ptr() if ws is not None else None, _lib.stream_ptr(x.device)),
        "pcb_quant_float8_dynamic",
    )
    if squeeze:
        data = data[0]
        if axiswise:
            scale = scale[0]
    return data, scale


# ------------------------------------------------------------------------ op ---
def _check_scale(scale: torch.Tensor, batch: int, rows: int, what: str) -> None:
    if scale.numel() != 1 and tuple(scale.shape) not in {(batch, rows), (batch, rows, 1)}:
        raise ValueError(f"{what} per-channel scale must have shape [B,{'M' if what == 'A' else 'N'}] or "
                         f"[B,{'M' if what == 'A' else 'N'},1], got {tuple(scale.shape)}")


def _bmm_linear_impl(a: torch.Tensor, b: torch.Tensor, scale_a: torch.Tensor, scale_b: torch.Tensor,
                     bias: torch.Tensor, use_bias: bool, output_dtype: torch.dtype,
                     per_channel: bool) -> torch.Tensor:
    batch, m, k = a.shape
    n = b.shape[-1]
    if b.shape[0] != batch or b.shape[1] != k:
        raise ValueError(f"incompatible BMM shapes: A={tuple(a.shape)}, B={tuple(b.shape)}")
    out = torch.empty((batch, m, n), device=a.device, dtype=output_dtype)
    # The op's scales are QUANT scales: out = acc / (sa * sb).  The kernel
    # multiplies by dequant factors, so pass their reciprocals.
    da = scale_a.float().reciprocal()
    db = scale_b.float().reciprocal()
    if per_channel and da.numel() != 1:
        da = da.reshape(batch, m)
        sa_strides = (da.stride(0), da.stride(1), 0)
    else:
        da = da.reshape(())
        sa_strides = (0, 0, 0)
    if per_channel and db.numel() != 1:
        db = db.reshape(batch, n)
        sb_strides = (db.stride(0), 0, db.stride(1))
    else:
        db = db.reshape(())
        sb_strides = (0, 0, 0)
    bias3 = None
    if use_bias:
        # [B, N] broadcast over M as a zero-stride view (stride_biasm = 0 in the reference).
        bias3 = bias.unsqueeze(1).expand(batch, m, n)
    return bmm_scaled(a, b, out, scale_a=da, sa_strides=sa_strides, qbm=1, scale_b=db, sb_strides=sb_strides,
                      qbn=1, qbk=max(k, 1), bias=bias3, activation="none")


@torch.library.custom_op("pcb200::bmm_linear_tma", mutates_args=())
def bmm_linear_tma(a: torch.Tensor, b: torch.Tensor, scale_a: torch.Tensor, scale_b: torch.Tensor,
                   bias: torch.Tensor, use_bias: bool, output_dtype: torch.dtype, per_channel: bool) -> torch.Tensor:
    """``fp8_bench::bmm_linear_tma`` (``bmm_linear.py:121-227``) on libpcb200:
    ``out[b] = (a[b] @ b[b]) / (scale_a * scale_b) + bias[b]`` in fp32,
    cast to ``output_dtype``.  ``a`` [B, M, K] fp8 (K- or M-major), ``b`` [B, K, N]
    fp8 (N- or K-major; its fp8 format may differ from ``a``'s); scales are
    the casts' quant scales, a single value or per channel ([B, M] / [B, N],
    optionally with a trailing 1); ``bias`` [B, N], read only if ``use_bias``."""
    return _bmm_linear_impl(a, b, scale_a, scale_b, bias, use_bias, output_dtype, per_channel)


@bmm_linear_tma.register_fake
def _(a, b, scale_a, scale_b, bias, use_bias, output_dtype, per_channel):
    return a.new_empty((a.shape[0], a.shape[1], b.shape[-1]), dtype=output_dtype)


def _fp8_bmm(a_data, a_scale, b_data, b_scale, output_dtype, bias=None) -> torch.Tensor:
    """``_fp8_bmm_tma`` (``bmm_linear.py:229-282``): shape checks, then the op."""
    if a_data.ndim != 3 or b_data.ndim != 3:
        raise ValueError(f"Float8 BMM expects rank-3 operands, got A={tuple(a_data.shape)}, B={tuple(b_data.shape)}")
    if a_data.shape[0] != b_data.shape[0] or a_data.shape[2] != b_data.shape[1]:
        raise ValueError(f"incompatible BMM shapes: A={tuple(a_data.shape)}, B={tuple(b_data.shape)}")
    if a_data.device != b_data.device or a_data.device.type != "cuda":
        raise ValueError("Float8 BMM operands must be CUDA tensors on the same device")
    batch, m, n = a_data.shape[0], a_data.shape[1], b_data.shape[2]
    per_channel = a_scale.numel() != 1 or b_scale.numel() != 1
    if per_channel:
        _check_scale(a_scale, batch, m, "A")
        _check_scale(b_scale, batch, n, "B")
    if bias is None:
        bias_arg, use_bias = a_data, False
    else:
        if bias.shape != (batch, n):
            raise ValueError(f"bias must have shape {(batch, n)}, got {tuple(bias.shape)}")
        bias_arg, use_bias = bias, True
    return bmm_linear_tma(a_data, b_data, a_scale, b_scale, bias_arg, use_bias, output_dtype, per_channel)


# ------------------------------------------------------------------ autograd ---
class _Float8BMMLinearFunction(torch.autograd.Function):
    """Forward ``Y = X W^T (+ bias)``, dgrad ``dX = dY W``, wgrad
    ``dW = dY^T X``, all three on the FP8 op (``bmm_linear.py:326-451``)."""

    @staticmethod
    def forward(ctx, input, weight, bias, config: Float8BMMLinearConfig):
        axis = config.scaling_granularity == "axiswise"
        x_data, x_scale = cast_to_float8(input, config.input_dtype, axis)
        w_data, w_scale = cast_to_float8(weight, config.weight_dtype, axis)
        ctx.save_for_backward(x_data, x_scale, w_data, w_scale)
        ctx.config = config
        ctx.has_bias = bias is not None
        ctx.in_dtype = input.dtype
        bias_k = None if bias is None else bias.to(input.dtype)
        # W [B, N, K] as the right operand [B, K, N]: a K-major view.
        return _fp8_bmm(x_data, x_scale, w_data.transpose(-2, -1), w_scale, input.dtype, bias_k)

    @staticmethod
    def backward(ctx, grad_output):
        x_data, x_scale, w_data, w_scale = ctx.saved_tensors
        config = ctx.config
        axis = config.scaling_granularity == "axiswise"
        batch, n = w_data.shape[0], w_data.shape[1]
        m = x_data.shape[1]
        if axis:
            # The weight's per-row quant scale becomes a reduction-dim scale
            # in dX: fold it into dY before the cast (bmm_linear.py:375-392).
            dy_hp = grad_output.to(torch.float32) / w_scale.reshape(batch, n).unsqueeze(1)
            dy_data, dy_scale = cast_to_float8(dy_hp, config.grad_output_dtype, True)
            w_b_scale = w_scale.new_ones(())
        else:
            dy_data, dy_scale = cast_to_float8(grad_output, config.grad_output_dtype, False)
            w_b_scale = w_scale
        grad_input = grad_weight = grad_bias = None
        if ctx.needs_input_grad[0]:
            # dX [B, M, K] = dY [B, M, N] @ W [B, N, K] (N-major right operand).
            grad_input = _fp8_bmm(dy_data, dy_scale, w_data, w_b_scale, grad_output.dtype)
        if ctx.needs_input_grad[1]:
            if axis:
                dyt_hp = grad_output.transpose(-2, -1).to(torch.float32) / x_scale.reshape(batch, m).unsqueeze(1)
                dyt_data, dyt_scale = cast_to_float8(dyt_hp, config.grad_output_dtype, True)
                x_b_scale = x_scale.new_ones(())
            else:
                dyt_data, dyt_scale = dy_data.transpose(-2, -1), dy_scale
                x_b_scale = x_scale
            # dW [B, N, K] = dY^T [B, N, M] @ X [B, M, K].
            grad_weight = _fp8_bmm(dyt_data, dyt_scale, x_data, x_b_scale, grad_output.dtype)
        if ctx.has_bias and ctx.needs_input_grad[2]:
            grad_bias = grad_output.sum(dim=1)
        return grad_input, grad_weight, grad_bias, None


# ------------------------------------------------------------------- modules ---
class BMMLinear(nn.Module):
    """High-precision batched dense layer (``bmm_linear.py:454-512``), the
    module :func:`convert_to_float8_bmm_training` replaces."""

    def __init__(self, batch_size: int, in_features: int, out_features: int, bias: bool = True, *,
                 device=None, dtype=None) -> None:
        super().__init__()
        if batch_size <= 0 or in_features <= 0 or out_features <= 0:
            raise ValueError("batch_size, in_features and out_features must be positive")
        self.batch_size, self.in_features, self.out_features = batch_size, in_features, out_features
        kw = {"device": device, "dtype": dtype}
        self.weight = nn.Parameter(torch.empty((batch_size, out_features, in_features), **kw))
        if bias:
            self.bias = nn.Parameter(torch.empty((batch_size, out_features), **kw))
        else:
            self.register_parameter("bias", None)
        self.reset_parameters()

    def reset_parameters(self) -> None:
        bound = 1 / math.sqrt(self.in_features)
        nn.init.uniform_(self.weight, -bound, bound)
        if self.bias is not None:
            nn.init.uniform_(self.bias, -bound, bound)

    def _check_input(self, input: torch.Tensor, name: str) -> None:
        if input.ndim != 3:
            raise ValueError(f"{name} expects [B,M,K], got {tuple(input.shape)}")
        if input.shape[0] != self.batch_size or input.shape[2] != self.in_features:
            raise ValueError("input shape mismatch: expected "
                             f"[{self.batch_size}, M, {self.in_features}], got {tuple(input.shape)}")

    def forward(self, input: torch.Tensor) -> torch.Tensor:
        self._check_input(input, "BMMLinear")
        out = torch.bmm(input, self.weight.transpose(-2, -1))
        if self.bias is not None:
            out = out + self.bias.unsqueeze(1)
        return out

    def extra_repr(self) -> str:
        return (f"batch_size={self.batch_size}, in_features={self.in_features}, "
                f"out_features={self.out_features}, bias={self.bias is not None}")


class Float8BMMLinear(BMMLinear):
    """Batched dense layer whose forward, dgrad and wgrad run as FP8 BMMs on
    libpcb200 (``Float8BMMLinear``, ``bmm_linear.py:515-660``).  ``config``:
    a :class:`Float8BMMLinearConfig` or the reference's config object."""

    def __init__(self, batch_size: int, in_features: int, out_features: int, bias: bool = True, *,
                 config=None, device=None, dtype=None) -> None:
        super().__init__(batch_size, in_features, out_features, bias, device=device, dtype=dtype)
        self.config = _resolve(config)

    def forward(self, input: torch.Tensor) -> torch.Tensor:
        self._check_input(input, "Float8BMMLinear")
        if torch.is_autocast_enabled():
            input = input.to(torch.get_autocast_gpu_dtype())
        return _Float8BMMLinearFunction.apply(input, self.weight, self.bias, self.config)

    def extra_repr(self) -> str:
        return (super().extra_repr() + f", backend=libpcb200_{self.config.scaling_granularity}, "
                f"fp8_all_gather={self.config.enable_fsdp_float8_all_gather}")

    @classmethod
    def from_float(cls, module: BMMLinear, config=None) -> "Float8BMMLinear":
        if not isinstance(module, BMMLinear):
            raise TypeError(f"expected BMMLinear, got {type(module)}")
        with torch.device("meta"):
            converted = cls(module.batch_size, module.in_features, module.out_features, bias=False)
        converted.config = _resolve(config)
        converted.weight = module.weight
        converted.bias = module.bias
        return converted


def convert_to_float8_bmm_training(module: nn.Module, config=None) -> nn.Module:
    """Recursively replace every :class:`BMMLinear` (or the reference's
    ``BMMLinear``, matched by class name and attributes) with its FP8 variant
    (``bmm_linear.py:661-673``)."""
    cfg = _resolve(config)

    def is_bmm_linear(m):
        return isinstance(m, BMMLinear) or (type(m).__name__ == "BMMLinear" and hasattr(m, "batch_size"))

    if is_bmm_linear(module) and not isinstance(module, Float8BMMLinear):
        if not isinstance(module, BMMLinear):
            plain = BMMLinear.__new__(BMMLinear)
            nn.Module.__init__(plain)
            plain.batch_size, plain.in_features, plain.out_features = (module.batch_size, module.in_features,
                                                                       module.out_features)
            plain.weight, plain.bias = module.weight, module.bias
            module = plain
        return Float8BMMLinear.from_float(module, cfg)
    for name, child in list(module.named_children()):
        new = convert_to_float8_bmm_training(child, cfg)
        if new is not child:
            module.register_module(name, new)
    return module


__all__ = [
    "BMMLinear",
    "Float8BMMLinear",
    "Float8BMMLinearConfig",
    "bmm_linear_tma",
    "cast_to_float8",
    "convert_to_float8_bmm_training",
]
