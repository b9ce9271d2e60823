"""CPU references for the scaled FP8 BMM (TEST INFRASTRUCTURE ONLY).

Three references, all fp32 on the CPU:

* ``scaled_bmm_dequant_reference`` -- the "kernel reference" of
  ``fp8_training/fp8_bench/bench_bmm.py:414-419``: dequantize both operands
  (``QuantResult.dequantize``), ``torch.bmm`` in fp32, add the bias, apply the
  epilogue activation (``kernels/bmm/activation.py:12-19``), cast.
* ``scaled_bmm_promoted_reference`` -- the per-K-group promotion order of
  ``kernels/bmm/per_block.py:99-111`` (fp32 partial of each K quant group,
  multiplied by ``sa * sb`` and added to an fp32 accumulator).  Closer to the
  kernel's rounding than the dequant reference; used for the tight checks.
* ``legacy_bmm_reference`` -- ``fp8_quant_bmm_ref`` of
  ``kernels/fp8_bmm/test/fp8_quant_bmm_test.py:100-114``.
"""

from __future__ import annotations

import math

import torch

from .quant import dequantize


def _activation(x: torch.Tensor, activation: str) -> torch.Tensor:
    if activation == "gelu":
        return 0.5 * x * (1.0 + torch.erf(x * 0.7071067811865475))
    if activation == "none":
        return x
    raise ValueError(f"activation must be 'none' or 'gelu', got {activation!r}")


def scaled_bmm_dequant_reference(
    a_q: torch.Tensor,
    a_scale: torch.Tensor,
    a_gran: str,
    a_meta: dict,
    b_q: torch.Tensor,
    b_scale: torch.Tensor,
    b_gran: str,
    b_meta: dict,
    *,
    bias: torch.Tensor | None = None,
    activation: str = "none",
    out_dtype: torch.dtype = torch.bfloat16,
) -> torch.Tensor:
    """fp32 ``bmm(dequant(A), dequant(B)) + bias`` -> activation -> cast."""
    a = dequantize(a_q.cpu(), a_scale.cpu(), a_gran, a_meta)
    b = dequantize(b_q.cpu(), b_scale.cpu(), b_gran, b_meta)
    acc = torch.bmm(a, b)
    if bias is not None:
        acc = acc + bias.cpu().float()
    return _activation(acc, activation).to(out_dtype)


def scaled_bmm_promoted_reference(
    a_q: torch.Tensor,
    a_scale: torch.Tensor,
    b_q: torch.Tensor,
    b_scale: torch.Tensor,
    *,
    qbm: int,
    qbk: int,
    qbn: int,
    bias: torch.Tensor | None = None,
    activation: str = "none",
    out_dtype: torch.dtype = torch.bfloat16,
) -> torch.Tensor:
    """Per-block BMM with the promotion order of ``kernels/bmm/per_block.py:99-111``.

    ``a_scale`` is ``[B, ceil(M/qbm), ceil(K/qbk)]`` and ``b_scale`` is
    ``[B, ceil(K/qbk), ceil(N/qbn)]``.
    """
    a = a_q.cpu().float()
    b = b_q.cpu().float()
    sa = a_scale.cpu().float()
    sb = b_scale.cpu().float()
    batch, m, k = a.shape
    n = b.shape[-1]
    rows = torch.arange(m) // qbm
    cols = torch.arange(n) // qbn
    acc = torch.zeros((batch, m, n), dtype=torch.float32)
    for g in range(math.ceil(k / qbk)):
        k0, k1 = g * qbk, min(k, (g + 1) * qbk)
        partial = torch.bmm(a[:, :, k0:k1], b[:, k0:k1, :])
        s = sa[:, :, g].index_select(1, rows)[:, :, None] * sb[:, g, :].index_select(1, cols)[:, None, :]
        acc += partial * s
    if bias is not None:
        acc = acc + bias.cpu().float()
    return _activation(acc, activation).to(out_dtype)


def legacy_bmm_reference(
    a: torch.Tensor,
    b: torch.Tensor,
    quant_scale,
    bias: torch.Tensor | None = None,
    out_dtype: torch.dtype = torch.bfloat16,
) -> torch.Tensor:
    """Exact fp32 matmul of fp8 inputs, times the scale, plus bias, cast."""
    acc = a.cpu().to(torch.float32) @ b.cpu().to(torch.float32)
    scale = quant_scale.cpu().to(torch.float32) if torch.is_tensor(quant_scale) else float(quant_scale)
    acc = acc * scale
    if bias is not None:
        acc = acc + bias.cpu().to(torch.float32)
    return acc.to(out_dtype)
