"""pcb_quant_per_tensor_noalloc: the per-tensor quantizer for callers that
cannot give the library any scratch memory (a plugin slot that only receives
its input and output tensors, or a loop that must not call cudaMalloc because
it can synchronise the device).  Its amax partials live in a fixed array
inside the library.  Called through the C ABI, its bytes and scales must equal
those of pcb_quant_per_tensor (the workspace-taking entry point) -- the same
bit-exact bar as every quantizer test -- on two calls in a row, the second on
a smaller tensor so that stale partials from the first call would show.

This file is named to be collected last."""

import pytest
import torch

from practice_cuda_b200 import _lib
from practice_cuda_b200.impls.b200_per_tensor import quantize_per_tensor
from tests._util import E4M3, assert_bytes_equal, assert_scales_equal, synthetic

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


def test_no_alloc_matches_workspace_entry_point():
    inputs = [
        synthetic((8, 1024, 2048), outliers=True, seed=101).cuda(),  # many amax CTAs, large amax
        synthetic((1, 33, 64), std=0.01, seed=102).cuda(),           # one CTA, small amax
    ]
    for i, x in enumerate(inputs):
        y_ref, q_ref, d_ref = quantize_per_tensor(x, E4M3, 448.0, 1e-12)
        y, q, d = _noalloc(x)
        torch.cuda.synchronize()
        assert_bytes_equal(y, y_ref, f"call {i} bytes")
        assert_scales_equal(q.reshape(1), q_ref.reshape(1), f"call {i} quant scale")
        assert_scales_equal(d.reshape(1), d_ref.reshape(1), f"call {i} dequant scale")
    assert _lib.device_error()[0] == 0
