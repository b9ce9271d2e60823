"""Per-block FP8 training linear (the FSDP2 FP8 training config).

``y = x @ w.T`` with all three GEMMs of a training step on the per-block FP8
path of libpcb200:

* forward  ``y  = q(x, 1x128 along in)  @ q(w, 128x128).T``
* dgrad    ``dx = q(dy, 1x128 along out) @ q(w, 128x128)``
* wgrad    ``dw = q(dy, 128x1 along tokens).T @ q(x, 128x1 along tokens)``

i.e. activations and gradients are scaled per 128 elements of the reduction
dimension of the GEMM that consumes them, weights per 128x128 tile (the
DeepSeek-V3 recipe).  This extends the reference's FP8 BMM linear
(``fp8_training/fp8_bench/modules/bmm_linear.py:326-451``, per-tensor /
per-channel only; its per-block module ``modules/per_block.py:13-118`` is
unfinished) to per-block scaling.  The weight ``w`` may arrive already
quantized (a :class:`BlockFP8Weight` produced by the FSDP2 FP8 all-gather in
``fsdp_fp8.py``), in which case the forward and dgrad reuse its fp8 bytes and
128x128 scales instead of re-quantizing.

Every quantization and GEMM is a libpcb200 kernel; the three GEMMs read the
operands in the layout autograd hands them (K-major / MN-major UMMA operands),
so no transposed copies are made.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from .impls.b200_per_block import b200_per_block_quant
from .impls._common import bmm_scaled

E4M3 = torch.float8_e4m3fn


class BlockFP8Weight(torch.Tensor):
    """An unsharded weight already quantized in 128x128 tiles.

    Wrapper subclass with the logical shape and dtype of the high-precision
    weight ([out, in], bf16) that carries ``data`` (fp8 [out, in]) and
    ``scale`` (fp32 [out/128, in/128]).  Only :class:`FP8BlockLinear` consumes
    it; it exists for the duration of one FSDP2 unshard.
    """

    @staticmethod
    def __new__(cls, data: torch.Tensor, scale: torch.Tensor, dtype: torch.dtype):
        return torch.Tensor._make_wrapper_subclass(
            cls, data.shape, dtype=dtype, device=data.device, requires_grad=False
        )

    def __init__(self, data: torch.Tensor, scale: torch.Tensor, dtype: torch.dtype):
        self._data = data
        self._scale = scale

    def __tensor_flatten__(self):
        return ["_data", "_scale"], {"dtype": self.dtype}

    @staticmethod
    def __tensor_unflatten__(inner, meta, outer_size, outer_stride):
        return BlockFP8Weight(inner["_data"], inner["_scale"], meta["dtype"])

    def __repr__(self):
        return f"BlockFP8Weight(shape={tuple(self.shape)}, dtype={self.dtype})"

    @classmethod
    def __torch_dispatch__(cls, func, types, args=(), kwargs=None):
        kwargs = kwargs or {}
        aten = torch.ops.aten
        w = args[0]
        if func in (aten.detach.default, aten.alias.default):
            return BlockFP8Weight(w._data, w._scale, w.dtype)
        if func in (aten.as_strided.default, aten.view.default, aten._unsafe_view.default, aten.reshape.default):
            if tuple(args[1]) != tuple(w.shape):
                raise NotImplementedError(f"BlockFP8Weight cannot be re-shaped by {func}")
            return BlockFP8Weight(w._data, w._scale, w.dtype)
        if func is aten.is_same_size.default:
            return tuple(args[0].shape) == tuple(args[1].shape)
        if func is aten._to_copy.default:
            # A dequantized high-precision copy (tests / debugging only).
            return dequantize_weight(w._data, w._scale).to(kwargs.get("dtype") or w.dtype)
        raise NotImplementedError(f"BlockFP8Weight does not support {func}")


def dequantize_weight(data: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    s = scale.repeat_interleave(128, 0)[: data.shape[0]].repeat_interleave(128, 1)[:, : data.shape[1]]
    return data.float() * s


def quantize_weight(w: torch.Tensor, pow2: bool = False) -> tuple[torch.Tensor, torch.Tensor]:
    """(fp8 [out, in], fp32 [out/128, in/128]) -- 128x128 tiles; ``pow2``
    selects power-of-two (E8M0) scales."""
    q = b200_per_block_quant(w, block_m=128, block_n=128, pow2_scales=pow2)
    return q.tensor, q.dequant_scale


def _as3(t: torch.Tensor) -> torch.Tensor:
    return t.unsqueeze(0)


def _gemm(a, a_scale, a_strides, qbm, b, b_scale, b_strides, qbn, out_dtype, block_scaled=False):
    """C[M, N] = sum_g (A_g B_g) sa sb with 128-deep K groups (2-D operands);
    ``block_scaled`` for power-of-two scales applied by the tensor core."""
    m = a.shape[0]
    n = b.shape[1]
    out = torch.empty((1, m, n), device=a.device, dtype=out_dtype)
    return bmm_scaled(
        _as3(a), _as3(b), out,
        scale_a=a_scale, sa_strides=(0,) + a_strides, qbm=qbm,
        scale_b=b_scale, sb_strides=(0,) + b_strides, qbn=qbn,
        qbk=128, bias=None, activation="none", block_scaled=block_scaled,
    )[0]


class _FP8BlockLinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x2d: torch.Tensor, weight: torch.Tensor, w_data, w_scale, pow2: bool = False):
        # x2d [T, in] bf16; weight is the high-precision parameter (for its
        # grad) and (w_data, w_scale) its 128x128 quantization.
        ctx.pow2 = pow2
        qx = b200_per_block_quant(x2d, block_m=1, block_n=128, pow2_scales=pow2)  # [T, in], scales [T, in/128]
        # y[T, out] = qx @ w.T: B = w.T is K-major (w stored [out, in]).
        wt = w_data.t()
        ws = w_scale
        y = _gemm(qx.tensor, qx.dequant_scale, tuple(qx.dequant_scale.stride()), 1,
                  wt, ws, (ws.stride(1), ws.stride(0)), 128, x2d.dtype, pow2)
        ctx.save_for_backward(x2d, w_data, w_scale)
        ctx.w_dtype = weight.dtype
        return y

    @staticmethod
    def backward(ctx, dy: torch.Tensor):
        x2d, w_data, w_scale = ctx.saved_tensors
        pow2 = ctx.pow2
        dy = dy.contiguous()
        # dgrad: dx[T, in] = q(dy 1x128 along out) @ w  (w as [K=out, N=in], N-major)
        qdy = b200_per_block_quant(dy, block_m=1, block_n=128, pow2_scales=pow2)
        dx = _gemm(qdy.tensor, qdy.dequant_scale, tuple(qdy.dequant_scale.stride()), 1,
                   w_data, w_scale, tuple(w_scale.stride()), 128, x2d.dtype, pow2)
        # wgrad: dw[out, in] = q(dy 128x1 along T).T @ q(x 128x1 along T)
        qdy_t = b200_per_block_quant(dy, block_m=128, block_n=1, pow2_scales=pow2)   # scales [T/128, out]
        qx_t = b200_per_block_quant(x2d, block_m=128, block_n=1, pow2_scales=pow2)   # scales [T/128, in]
        a = qdy_t.tensor.t()                                       # [out, T], M-major
        sa = qdy_t.dequant_scale                                   # [T/128, out] -> (m, kg)
        b = qx_t.tensor                                            # [T, in], N-major
        sb = qx_t.dequant_scale                                    # [T/128, in] -> (kg, n)
        dw = _gemm(a, sa, (sa.stride(1), sa.stride(0)), 1, b, sb, tuple(sb.stride()), 1, ctx.w_dtype, pow2)
        return dx, dw, None, None, None


class FP8BlockLinear(nn.Linear):
    """``nn.Linear`` whose forward, dgrad and wgrad run on the per-block FP8
    kernels (bias, if any, is added in high precision).

    ``scaling`` (attribute, default ``"fp32"``): ``"fp32"`` quantizes with the
    reference's fp32 scales (``dequant = 1 / (448 / amax)``) and promotes each
    128-deep K group in the GEMM epilogue; ``"e8m0"`` rounds every scale up
    to a power of two so the tensor core applies it
    (``pcb_bmm_block_scaled``) and the accumulator never leaves TMEM.
    """

    scaling: str = "fp32"

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        w = self.weight
        if isinstance(w, BlockFP8Weight):  # unsharded by the FSDP2 FP8 all-gather
            w_data, w_scale = w._data, w._scale
        else:
            master = getattr(w, "_tensor", w)  # FP8AllGatherWeight outside FSDP: its plain tensor
            w_data, w_scale = quantize_weight(master.detach(), pow2=self.scaling == "e8m0")
        w_hp = w
        shape = x.shape
        x2d = x.reshape(-1, shape[-1])
        if x2d.stride(-1) != 1:
            x2d = x2d.contiguous()
        y = _FP8BlockLinearFn.apply(x2d, w_hp, w_data, w_scale, self.scaling == "e8m0")
        y = y.reshape(*shape[:-1], y.shape[-1])
        if self.bias is not None:
            y = y + self.bias
        return y


def convert_to_fp8_block_linear(module: nn.Module, *, skip=lambda name, m: False, scaling: str = "fp32") -> nn.Module:
    """Swap every ``nn.Linear`` (except those ``skip`` selects) for an
    :class:`FP8BlockLinear` sharing its parameters (cf. the reference's
    ``convert_to_float8_bmm_training``, ``modules/bmm_linear.py:661-673``)."""
    for name, child in list(module.named_children()):
        if isinstance(child, nn.Linear) and not isinstance(child, FP8BlockLinear) and not skip(name, child):
            new = FP8BlockLinear.__new__(FP8BlockLinear)
            nn.Module.__init__(new)
            new.in_features, new.out_features = child.in_features, child.out_features
            new.weight = child.weight
            new.bias = child.bias
            new.scaling = scaling
            setattr(module, name, new)
        else:
            convert_to_fp8_block_linear(child, skip=skip, scaling=scaling)
    return module
