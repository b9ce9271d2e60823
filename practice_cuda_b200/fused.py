"""Fused quantize -> scaled FP8 GEMM (BASELINE cfg4).

``quant_bmm_fused(x, qb)`` quantizes the bf16/fp16 activation ``x`` in 1x128
groups inside the GEMM kernel (pcb_quant_bmm_fused) and multiplies it by the
pre-quantized per-block (or per-channel) weight ``qb``.  It is what the
reference's non-functional fused kernel
(``kernels/fp8_bmm/kernel/fp8_quant_bmm_fused_kernel.py:39-146``) set out to
do, with the numerics of the unfused pipeline
``b200_per_block_quant(x, 1, 128)`` + ``b200_per_block_bmm``: the quantized
activation is bit-identical and the output matches within the GEMM tolerance.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import _lib
from .impls._common import pack_k_major
from .registry import QuantResult


def quant_bmm_fused(
    x: torch.Tensor,
    b: QuantResult,
    *,
    out_dtype: torch.dtype = torch.bfloat16,
    bias: Optional[torch.Tensor] = None,
    out: Optional[torch.Tensor] = None,
    activation: str = "none",
    eps: float = 1e-12,
    return_quantized: bool = False,
    fuse: Optional[bool] = None,
):
    """``act(quant_1x128(x) @ b + bias)``.

    The fused kernel quantizes each 128x128 activation tile inside every
    output tile that consumes it, so its quantization work grows with the
    number of 128-wide output column blocks.  ``fuse=None`` (default) uses it
    when N <= 256 (at most two column blocks) and otherwise runs the 1x128
    quantizer once followed by the per-block GEMM (two launches, identical
    results); ``fuse=True`` / ``False`` forces either path.  ``x`` is [B, M, K] (or [M, K]),
    K contiguous; ``b`` is an e4m3 QuantResult [B, K, N] with 128-deep K blocks.
    With ``return_quantized`` also returns the QuantResult of ``x``."""
    if activation not in ("none", "gelu"):
        raise ValueError(f"activation must be 'none' or 'gelu', got {activation!r}")
    squeeze = x.ndim == 2
    if squeeze:
        x = x.unsqueeze(0)
    if x.ndim != 3 or b.tensor.ndim != 3:
        raise ValueError("fused BMM expects a 2D/3D activation and a 3D quantized B")
    _lib.require_cuda(x, "x")
    if x.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError(f"x must be bfloat16 or float16, got {x.dtype}")
    if b.tensor.dtype != torch.float8_e4m3fn:
        raise ValueError(f"B must be float8_e4m3fn, got {b.tensor.dtype}")
    if x.stride(-1) != 1:
        x = x.contiguous()
    batch, m, k = x.shape
    bb, bk, n = b.tensor.shape
    if bb != batch or bk != k:
        raise ValueError(f"shape mismatch: x={tuple(x.shape)}, B={tuple(b.tensor.shape)}")
    sb = b.dequant_scale
    if b.granularity == "block":
        if b.meta.get("block_m") != 128:
            raise ValueError(f"B must be quantized with block_m=128 (the K block), got {b.meta.get('block_m')}")
        qbn = b.meta["block_n"]
        sb_strides = (sb.stride(0), sb.stride(1), sb.stride(2))
        if tuple(sb.shape) != (batch, (k + 127) // 128, (n + qbn - 1) // qbn):
            raise ValueError(f"B dequant scale has shape {tuple(sb.shape)}")
    elif b.granularity == "channel" and b.meta.get("channel_axis") == -1:
        qbn = 1
        sb_strides = (sb.stride(0), 0, sb.stride(1))
    else:
        raise ValueError("B must be per-block (128 x block_n) or per-channel (channel_axis=-1)")
    if out is None:
        out = torch.empty((batch, m, n), device=x.device, dtype=out_dtype)
    if fuse is None:
        fuse = n <= 256
    if not fuse:
        from .impls.b200_per_block import b200_per_block_bmm, b200_per_block_quant

        qx = b200_per_block_quant(x, block_m=1, block_n=128, eps=eps)
        if b.granularity == "block":
            b200_per_block_bmm(qx, b, out_dtype=out_dtype, bias=bias, out=out, activation=activation)
        else:
            # per-channel B with 1x128 A: per-block BMM with a 128 x 1 view of the B scales
            bscale = sb.unsqueeze(1).expand(batch, (k + 127) // 128, n).contiguous()
            qb2 = QuantResult(b.tensor, bscale, b.impl, "block", {"block_m": 128, "block_n": 1})
            b200_per_block_bmm(qx, qb2, out_dtype=out_dtype, bias=bias, out=out, activation=activation)
        if squeeze:
            out = out[0]
            qx = QuantResult(qx.tensor[0], qx.dequant_scale[0], qx.impl, qx.granularity, dict(qx.meta))
        return (out, qx) if return_quantized else out
    if bias is not None and bias.shape != (batch, m, n):
        raise ValueError(f"bias must have shape {(batch, m, n)}, got {tuple(bias.shape)}")
    xq = xs = None
    if return_quantized:
        xq = torch.empty((batch, m, k), device=x.device, dtype=torch.float8_e4m3fn)
        xs = torch.empty((batch, m, (k + 127) // 128), device=x.device, dtype=torch.float32)
    lib = _lib.lib()

    def launch(bt):
        return lib.pcb_quant_bmm_fused(
            x.data_ptr(), _lib.dtype_code(x.dtype), *x.stride(),
            bt.data_ptr(), *bt.stride(), _lib.dtype_code(bt.dtype),
            batch, m, n, k,
            sb.data_ptr(), *sb_strides, qbn,
            bias.data_ptr() if bias is not None else None,
            _lib.dtype_code(bias.dtype) if bias is not None else 0,
            *(bias.stride() if bias is not None else (0, 0, 0)),
            out.data_ptr(), _lib.dtype_code(out.dtype), *out.stride(),
            xq.data_ptr() if xq is not None else None, *(xq.stride()[:2] if xq is not None else (0, 0)),
            xs.data_ptr() if xs is not None else None, *(xs.stride() if xs is not None else (0, 0, 0)),
            _lib.PCB_ACT[activation], eps, _lib.stream_ptr(x.device),
        )

    status = launch(b.tensor)
    if status == _lib.PCB_ERR_LAYOUT:  # B strides TMA cannot address: K-major, 16-byte padded copy
        status = launch(pack_k_major(b.tensor, k_dim_last=False))
    _lib.check(status, "pcb_quant_bmm_fused")
    if squeeze:
        out = out[0]
    if not return_quantized:
        return out
    qx = QuantResult(xq[0] if squeeze else xq, xs[0] if squeeze else xs, "b200_fused", "block",
                     {"logical_shape": tuple(x.shape), "fp8_dtype": str(torch.float8_e4m3fn),
                      "block_m": 1, "block_n": 128})
    return out, qx
