"""Shared host logic of the impl wrappers: layout detection with the
reference's error messages, output/bias validation, and the call into
pcb_bmm_scaled with in-call repacking of operands whose strides TMA cannot
address (the role of the reference's do_transpose_a / do_transpose_b
packing, ``fp8_training/fp8_bench/impls/triton_per_block.py:254-275``)."""

from __future__ import annotations

from typing import Optional

import torch

from .. import _lib


def matrix_layout(tensor: torch.Tensor, name: str) -> str:
    """``_matrix_layout`` of ``impls/triton_per_block.py:34-42``."""
    if tensor.stride(-1) == 1:
        return "n-major"
    if tensor.stride(-2) == 1:
        return "k-major"
    raise ValueError(
        f"{name} must be contiguous along one matrix dimension; "
        f"shape={tuple(tensor.shape)}, strides={tensor.stride()}"
    )


def a_layout(tensor: torch.Tensor) -> str:
    """``_a_layout`` of ``impls/triton_per_block.py:45-53``."""
    if tensor.stride(-1) == 1:
        return "k-major"
    if tensor.stride(-2) == 1:
        return "m-major"
    raise ValueError(
        "A must be contiguous along either K or M; "
        f"shape={tuple(tensor.shape)}, strides={tensor.stride()}"
    )


def is_power_of_two(value: int) -> bool:
    return value > 0 and (value & (value - 1)) == 0


def check_activation(activation: str) -> None:
    if activation not in ("none", "gelu"):
        raise ValueError(f"activation must be 'none' or 'gelu', got {activation!r}")


def resolve_operands(a: torch.Tensor, b: torch.Tensor, do_transpose_a: bool, do_transpose_b: bool):
    """Apply the reference's transpose/packing flags (triton_per_block.py:254-275)."""
    input_a_layout = a_layout(a)
    if do_transpose_a:
        if input_a_layout != "m-major":
            raise ValueError(f"do_transpose_a=True requires an M-major A input; strides={a.stride()}")
        a = pack_k_major(a, k_dim_last=True)
    input_b_layout = matrix_layout(b, "B")
    if do_transpose_b:
        if input_b_layout != "n-major":
            raise ValueError(f"do_transpose_b=True requires an N-major B input; strides={b.stride()}")
        b = pack_k_major(b, k_dim_last=False)
    batch, m, k = a.shape
    b_batch, b_k, n = b.shape
    if batch != b_batch or k != b_k:
        raise ValueError(f"shape mismatch: A={tuple(a.shape)}, B={tuple(b.shape)}")
    if a.device != b.device:
        raise ValueError(f"A and B must be on the same device: A={a.device}, B={b.device}")
    if a.dtype != b.dtype:
        raise ValueError(f"A and B must have the same FP8 dtype: A={a.dtype}, B={b.dtype}")
    return a, b


def pack_k_major(t: torch.Tensor, *, k_dim_last: bool) -> torch.Tensor:
    """Copy an fp8 operand into K-major storage with K padded to 16 bytes.

    ``k_dim_last`` is True for A ([B, M, K], K is dim -1) and False for B
    ([B, K, N], K is dim -2).  Returns a view with the logical shape of ``t``.
    """
    batch = t.shape[0]
    if k_dim_last:
        rows, cols = t.shape[1], t.shape[2]
        ssr, ssc = t.stride(1), t.stride(2)
    else:
        rows, cols = t.shape[2], t.shape[1]
        ssr, ssc = t.stride(2), t.stride(1)
    kp = max(16, (cols + 15) // 16 * 16)
    buf = torch.empty((batch, rows, kp), dtype=t.dtype, device=t.device)
    _lib.check(
        _lib.lib().pcb_pack_u8(t.data_ptr(), batch, rows, cols, t.stride(0), ssr, ssc,
                               buf.data_ptr(), rows * kp, kp, kp, _lib.stream_ptr(t.device)),
        "pcb_pack_u8",
    )
    view = buf[:, :, :cols]
    return view if k_dim_last else view.transpose(1, 2)


def check_out(out: Optional[torch.Tensor], batch: int, m: int, n: int, device, out_dtype) -> torch.Tensor:
    """Output allocation / validation of triton_per_block.py:326-341."""
    if out is None:
        return torch.empty((batch, m, n), device=device, dtype=out_dtype)
    if out.shape != (batch, m, n):
        raise ValueError(f"out must have shape {(batch, m, n)}, got {tuple(out.shape)}")
    if out.device != device:
        raise ValueError(f"out must be on {device}, got {out.device}")
    if out.dtype != out_dtype:
        raise ValueError(f"out must have dtype {out_dtype}, got {out.dtype}")
    if out.stride(-1) != 1:
        raise ValueError(f"out must be contiguous along N; shape={tuple(out.shape)}, strides={out.stride()}")
    return out


def check_bias(bias: Optional[torch.Tensor], batch: int, m: int, n: int, device, require_n_contiguous: bool):
    if bias is None:
        return
    if bias.shape != (batch, m, n):
        raise ValueError(f"bias must have shape {(batch, m, n)}, got {tuple(bias.shape)}")
    if bias.device != device:
        raise ValueError(f"bias must be on {device}, got {bias.device}")
    if require_n_contiguous and bias.stride(-1) != 1:
        raise ValueError(f"bias must be contiguous along N; shape={tuple(bias.shape)}, strides={bias.stride()}")


def bmm_scaled(
    a: torch.Tensor,
    b: torch.Tensor,
    out: torch.Tensor,
    *,
    scale_a: Optional[torch.Tensor],
    sa_strides: tuple[int, int, int],
    qbm: int,
    scale_b: Optional[torch.Tensor],
    sb_strides: tuple[int, int, int],
    qbn: int,
    qbk: int,
    bias: Optional[torch.Tensor],
    activation: str,
    block_scaled: bool = False,
) -> torch.Tensor:
    """Launch pcb_bmm_scaled (pcb_bmm_block_scaled for power-of-two scales
    applied by the tensor core); repack A/B to K-major once if TMA rejects them."""
    _lib.require_cuda(a, "A")
    batch, m, k = a.shape
    n = b.shape[-1]
    lib = _lib.lib()
    stream = _lib.stream_ptr(a.device)

    entry = lib.pcb_bmm_block_scaled if block_scaled else lib.pcb_bmm_scaled
    tail = (stream,)
    if block_scaled:
        ws_bytes = lib.pcb_bmm_block_scaled_workspace_bytes(batch, m, n, k)
        workspace = torch.empty((max(ws_bytes, 16),), dtype=torch.uint8, device=a.device)
        tail = (workspace.data_ptr(), ws_bytes, stream)

    mixed = a.dtype != b.dtype
    if mixed and block_scaled:
        raise ValueError(f"block-scaled BMM needs one fp8 format, got A={a.dtype}, B={b.dtype}")
    if mixed:
        entry = lib.pcb_bmm_scaled_mixed

    def launch(a_t, b_t):
        if mixed:
            head = (a_t.data_ptr(), a_t.stride(0), a_t.stride(1), a_t.stride(2), _lib.dtype_code(a_t.dtype),
                    b_t.data_ptr(), b_t.stride(0), b_t.stride(1), b_t.stride(2), _lib.dtype_code(b_t.dtype))
        else:
            head = (a_t.data_ptr(), a_t.stride(0), a_t.stride(1), a_t.stride(2),
                    b_t.data_ptr(), b_t.stride(0), b_t.stride(1), b_t.stride(2), _lib.dtype_code(a_t.dtype))
        return entry(
            *head,
            batch, m, n, k,
            scale_a.data_ptr() if scale_a is not None else None, *sa_strides, qbm,
            scale_b.data_ptr() if scale_b is not None else None, *sb_strides, qbn,
            qbk,
            bias.data_ptr() if bias is not None else None,
            _lib.dtype_code(bias.dtype) if bias is not None else 0,
            *(bias.stride() if bias is not None else (0, 0, 0)),
            out.data_ptr(), _lib.dtype_code(out.dtype), out.stride(0), out.stride(1), out.stride(2),
            _lib.PCB_ACT[activation], *tail,
        )

    status = launch(a, b)
    if status == _lib.PCB_ERR_LAYOUT and k > 0:
        status = launch(pack_k_major(a, k_dim_last=True), pack_k_major(b, k_dim_last=False))
    _lib.check(status, "pcb_bmm_block_scaled" if block_scaled else ("pcb_bmm_scaled_mixed" if mixed else "pcb_bmm_scaled"))
    return out
