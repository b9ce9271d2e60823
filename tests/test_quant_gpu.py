"""Quantization kernels vs the CPU oracle: bit-exact bytes and scales."""

import pytest
import torch

import oracle
from practice_cuda_b200 import get_quant
from practice_cuda_b200.impls.b200_per_channel import per_channel_quant_torch_compile
from tests._util import E4M3, E5M2, assert_bytes_equal, assert_scales_equal, synthetic

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _per_block(x, bm, bn, fp8=E4M3):
    return get_quant("b200_per_block_2d").fn(x.to(DEV), block_m=bm, block_n=bn, fp8_dtype=fp8)


def test_golden_per_block(golden):
    for name, c in golden.items():
        if c["kind"] != "per_block":
            continue
        q = _per_block(c["x"], c["block_m"], c["block_n"])
        assert_bytes_equal(q.tensor, c["y_u8"], name)
        assert_scales_equal(q.dequant_scale, c["scale"], name)


def test_golden_per_channel(golden):
    for name, c in golden.items():
        if c["kind"] != "per_channel":
            continue
        q = get_quant("b200_per_channel").fn(c["x"].to(DEV), channel_axis=c["channel_axis"])
        assert_bytes_equal(q.tensor, c["y_u8"], name)
        assert_scales_equal(q.dequant_scale, c["scale"], name)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.float16])
@pytest.mark.parametrize("shape,bm,bn", [
    ((4, 70, 384), 1, 128),
    ((2, 300, 264), 128, 128),
    ((257, 136), 128, 128),
    ((3, 33, 200), 1, 128),
    ((64, 512), 64, 32),
    ((2, 256, 96), 128, 1),
    ((96, 1024), 1, 1024),
])
def test_per_block_vs_oracle(dtype, shape, bm, bn):
    x = synthetic(shape, outliers=True, seed=hash((shape, bm, bn)) % 1000, dtype=dtype)
    q = _per_block(x, bm, bn)
    y_ref, s_ref = oracle.per_block_quant(x, block_m=bm, block_n=bn)
    assert_bytes_equal(q.tensor, y_ref, f"{shape} {bm}x{bn} {dtype}")
    assert_scales_equal(q.dequant_scale, s_ref, f"{shape} {bm}x{bn} {dtype}")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_per_block_128x128_strided_rows_and_many_tiles(dtype):
    """128x128 tiles of a column-sliced view (row stride > n) and a tensor with
    many more tiles than SMs, so every CTA's staging ring wraps several times."""
    base = synthetic((3, 300, 392), outliers=True, seed=31, dtype=dtype)
    x = base.to(DEV)[:, :, :264]
    assert x.stride(1) == 392
    q = _per_block(x, 128, 128)
    y_ref, s_ref = oracle.per_block_quant(base[:, :, :264].contiguous(), block_m=128, block_n=128)
    assert_bytes_equal(q.tensor, y_ref, f"strided {dtype}")
    assert_scales_equal(q.dequant_scale, s_ref, f"strided {dtype}")
    big = synthetic((6, 1024, 2048), seed=32, dtype=dtype)
    q = _per_block(big, 128, 128)
    y_ref, s_ref = oracle.per_block_quant(big, block_m=128, block_n=128)
    assert_bytes_equal(q.tensor, y_ref, f"many tiles {dtype}")
    assert_scales_equal(q.dequant_scale, s_ref, f"many tiles {dtype}")


def test_per_block_cfg1_full_size():
    """BASELINE cfg1 at full size: x [4096,7168] 1x128 and w [7168,7168] 128x128."""
    x = synthetic((4096, 7168), outliers=True, seed=0)
    q = _per_block(x, 1, 128)
    y_ref, s_ref = oracle.per_block_quant(x, block_m=1, block_n=128)
    assert q.dequant_scale.shape == (4096, 56)
    assert_bytes_equal(q.tensor, y_ref, "cfg1 x")
    assert_scales_equal(q.dequant_scale, s_ref, "cfg1 x")
    w = synthetic((7168, 7168), std=0.02, seed=1)
    q = _per_block(w, 128, 128)
    y_ref, s_ref = oracle.per_block_quant(w, block_m=128, block_n=128)
    assert q.dequant_scale.shape == (56, 56)
    assert_bytes_equal(q.tensor, y_ref, "cfg1 w")
    assert_scales_equal(q.dequant_scale, s_ref, "cfg1 w")


def test_per_block_strided_input_generic_path():
    x = synthetic((2, 200, 160), seed=5)
    xt = x.transpose(1, 2)  # non-contiguous along n -> generic kernel
    q = _per_block(xt, 1, 128)
    y_ref, s_ref = oracle.per_block_quant(xt.contiguous(), block_m=1, block_n=128)
    assert_bytes_equal(q.tensor, y_ref, "strided")
    assert_scales_equal(q.dequant_scale, s_ref, "strided")


def test_per_block_e5m2():
    x = synthetic((64, 256), outliers=True, seed=6)
    q = _per_block(x, 1, 128, fp8=E5M2)
    y_ref, s_ref = oracle.per_block_quant(x, block_m=1, block_n=128, fp8_dtype=E5M2)
    assert q.tensor.dtype == E5M2
    assert_bytes_equal(q.tensor, y_ref, "e5m2")
    assert_scales_equal(q.dequant_scale, s_ref, "e5m2")


def test_per_block_zeros_and_outliers():
    x = torch.zeros((4, 256), dtype=torch.bfloat16)
    x[1, 3] = 1e6
    x[2, 130] = -1e6
    q = _per_block(x, 1, 128)
    y_ref, s_ref = oracle.per_block_quant(x, block_m=1, block_n=128)
    assert_bytes_equal(q.tensor, y_ref, "zeros/outliers")
    assert_scales_equal(q.dequant_scale, s_ref, "zeros/outliers")
    assert torch.isfinite(q.dequant_scale).all()


@pytest.mark.parametrize("axis", [-2, -1])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("shape", [(8192, 4096), (3, 33, 200), (2, 1000, 72), (5000, 16), (16, 20000)])
def test_per_channel_vs_oracle(axis, dtype, shape):
    if shape == (8192, 4096) and dtype == torch.float32:
        pytest.skip("cfg2 size covered in bf16")
    x = synthetic(shape, outliers=True, seed=len(shape) + axis, dtype=dtype)
    q = get_quant("b200_per_channel").fn(x.to(DEV), channel_axis=axis)
    y_ref, s_ref = oracle.per_channel_quant(x, channel_axis=axis)
    assert_bytes_equal(q.tensor, y_ref, f"{shape} axis={axis}")
    assert_scales_equal(q.dequant_scale, s_ref, f"{shape} axis={axis}")


def test_per_channel_column_major_input():
    x = synthetic((3, 96, 40), seed=9)
    xc = x.transpose(1, 2).contiguous().transpose(1, 2)  # stride(-2) == 1
    for axis in (-1, -2):
        q = get_quant("b200_per_channel").fn(xc.to(DEV), channel_axis=axis)
        y_ref, s_ref = oracle.per_channel_quant(x, channel_axis=axis)
        assert q.tensor.stride() == xc.stride()
        assert_bytes_equal(q.tensor.contiguous(), y_ref, f"col-major axis={axis}")
        assert_scales_equal(q.dequant_scale, s_ref, f"col-major axis={axis}")


def test_per_channel_torch_compile_signature():
    x = synthetic((64, 128), seed=10)
    y, s = per_channel_quant_torch_compile(x.to(DEV), -2, E4M3, 1e-12)
    y_ref, s_ref = oracle.per_channel_quant(x, channel_axis=-2)
    assert_bytes_equal(y, y_ref)
    assert_scales_equal(s, s_ref)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.float16])
@pytest.mark.parametrize("shape", [(128, 256), (17, 33), (3, 2048, 960)])
def test_per_tensor_vs_oracle(dtype, shape):
    x = synthetic(shape, outliers=True, seed=11, dtype=dtype)
    q = get_quant("b200_per_tensor").fn(x.to(DEV))
    y_ref, s_ref = oracle.per_tensor_quant(x)
    assert_bytes_equal(q.tensor, y_ref, f"{shape} {dtype}")
    assert_scales_equal(q.dequant_scale.reshape(()), s_ref.reshape(()), f"{shape} {dtype}")


def test_dequantize_roundtrip_block():
    x = synthetic((2, 64, 256), seed=12)
    q = _per_block(x, 1, 128)
    xh = q.dequantize().cpu()
    amax = x.float().abs().amax().item()
    assert torch.allclose(xh, x.float(), rtol=0.1, atol=0.05 * amax)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("shape,bm,bn", [
    ((2, 300, 264), 1, 128),
    ((2, 300, 264), 128, 128),
    ((3, 384, 136), 128, 1),
    ((257, 1024), 1, 128),
])
def test_per_block_pow2_vs_oracle(dtype, shape, bm, bn):
    """Power-of-two (E8M0) scales of the training recipe: bytes and scales
    bit-exact against the oracle restatement, every scale a power of two."""
    x = synthetic(shape, outliers=True, seed=hash((shape, bm, bn, 2)) % 1000, dtype=dtype)
    x[..., 0, :] = 0  # an all-zero row hits the eps clamp
    q = get_quant("b200_per_block_2d").fn(x.to(DEV), block_m=bm, block_n=bn, pow2_scales=True)
    y_ref, s_ref = oracle.per_block_quant_pow2(x, block_m=bm, block_n=bn)
    assert_bytes_equal(q.tensor, y_ref, f"pow2 {shape} {bm}x{bn} {dtype}")
    assert_scales_equal(q.dequant_scale, s_ref, f"pow2 {shape} {bm}x{bn} {dtype}")
    s = q.dequant_scale.cpu()
    assert torch.equal(torch.frexp(s).mantissa, torch.full_like(s, 0.5))
    assert q.meta["scale_format"] == "e8m0"


# Per-channel rows through the one-warp-per-row kernel (rows of up to 512
# 16-byte chunks) and the CTA-per-row kernel beyond: every input dtype, both
# fp8 formats, row counts that leave a partial CTA, a batched (3-D) input,
# an all-zero row.
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("fp8", [E4M3, E5M2])
@pytest.mark.parametrize("shape", [(13, 512), (1001, 4096), (3, 77, 2048), (64, 1000), (9, 8192)])
def test_per_channel_rows_vs_oracle(dtype, fp8, shape):
    es = torch.tensor([], dtype=dtype).element_size()
    if shape[-1] * es > 8192 and dtype != torch.bfloat16:
        pytest.skip("one length beyond 512 chunks is enough")
    x = synthetic(shape, dtype=dtype, outliers=True, seed=7)
    x[..., 3, :] = 0  # an all-zero row: amax clamps to eps
    q = get_quant("b200_per_channel").fn(x.to(DEV), channel_axis=-2, fp8_dtype=fp8)
    y_ref, s_ref = oracle.per_channel_quant(x, channel_axis=-2, fp8_dtype=fp8)
    assert_bytes_equal(q.tensor, y_ref, f"rows {dtype} {shape}")
    assert_scales_equal(q.dequant_scale, s_ref, f"rows scales {dtype} {shape}")
