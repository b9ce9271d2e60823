"""pcb_quant_per_tensor_noalloc: the per-tensor quantizer for callers that
cannot give the library any scratch memory (a plugin slot that only receives
its input and output tensors, or a loop that must not call cudaMalloc because
it can synchronise the device).  Its amax partials live in a fixed array
inside the library.  Called through the C ABI, its bytes and scales must equal
those of pcb_quant_per_tensor (the workspace-taking entry point) and of the
CPU oracle -- the same bit-exact bar as every quantizer test -- on two calls
in a row, the second on a smaller tensor so that stale partials from the
first call would show, for contiguous and strided bf16, fp16 and E5M2.

This file is named to be collected last."""

import pytest
import torch

import oracle
from practice_cuda_b200 import _lib
from practice_cuda_b200.impls.b200_per_tensor import quantize_per_tensor
from tests._util import E4M3, E5M2, assert_bytes_equal, assert_scales_equal, synthetic

pytestmark = pytest.mark.gpu


def _noalloc(x: torch.Tensor, fp8_dtype=E4M3, fp8_max=448.0, eps=1e-12):
    y = torch.empty_like(x, dtype=fp8_dtype)
    scales = torch.empty(2, device=x.device, dtype=torch.float32)
    batch, m, n = x.shape
    lib = _lib.lib()
    st = lib.pcb_quant_per_tensor_noalloc(
        x.data_ptr(), _lib.dtype_code(x.dtype), batch, m, n, *x.stride(),
        y.data_ptr(), _lib.dtype_code(fp8_dtype), *y.stride(),
        scales[0:1].data_ptr(), scales[1:2].data_ptr(), _lib.dtype_code(torch.float32), fp8_max, eps,
        _lib.stream_ptr(x.device))
    _lib.check(st, "pcb_quant_per_tensor_noalloc")
    return y, scales[0], scales[1]


def _variant(x: torch.Tensor, variant: str) -> torch.Tensor:
    """The same values laid out / typed for one launch path of the quantizer."""
    if variant == "strided":  # not contiguous along n: the scalar (non-vector) grid sizing
        return x.transpose(-1, -2).contiguous().transpose(-1, -2)
    if variant == "fp16":
        return x.to(torch.float16)
    return x


@pytest.mark.parametrize("variant,fp8_dtype", [
    ("contiguous", E4M3),
    ("strided", E4M3),
    ("fp16", E4M3),
    ("contiguous", E5M2),
])
def test_no_alloc_matches_workspace_entry_point_and_oracle(variant, fp8_dtype):
    fp8_max = 448.0 if fp8_dtype == E4M3 else 57344.0
    inputs = [
        synthetic((8, 1024, 2048), outliers=True, seed=101),  # many amax CTAs, large amax
        synthetic((1, 33, 64), std=0.01, seed=102),           # one CTA, small amax
    ]
    for i, x_cpu in enumerate(inputs):  # two calls in a row: stale partials of the first would show
        x = _variant(x_cpu.cuda(), variant)
        y_ref, q_ref, d_ref = quantize_per_tensor(x, fp8_dtype, fp8_max, 1e-12)
        y, q, d = _noalloc(x, fp8_dtype, fp8_max)
        torch.cuda.synchronize()
        what = f"{variant} {fp8_dtype} call {i}"
        assert_bytes_equal(y, y_ref, f"{what} bytes")
        assert_scales_equal(q.reshape(1), q_ref.reshape(1), f"{what} quant scale")
        assert_scales_equal(d.reshape(1), d_ref.reshape(1), f"{what} dequant scale")
        # and the CPU oracle (the reference's per-tensor formula) on the same values
        y_o, d_o = oracle.per_tensor_quant(x.cpu(), fp8_dtype=fp8_dtype)
        assert_bytes_equal(y, y_o, f"{what} bytes vs oracle")
        assert_scales_equal(d.reshape(1), d_o.reshape(1), f"{what} dequant scale vs oracle")
    assert _lib.device_error()[0] == 0
