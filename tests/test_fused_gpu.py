"""Fused quantize -> GEMM vs the unfused pipeline and the CPU oracle."""

import pytest
import torch

import oracle
from practice_cuda_b200 import get_quant
from practice_cuda_b200.fused import quant_bmm_fused
from tests._util import assert_bmm_close, assert_bytes_equal, assert_scales_equal, synthetic

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("shape", [(1, 256, 512, 384), (2, 200, 264, 136), (1, 128, 128, 128)])
@pytest.mark.parametrize("b_layout", ["n", "k"])
@pytest.mark.parametrize("fuse", [True, False])
def test_fused_matches_oracle(shape, b_layout, fuse):
    B, M, K, N = shape
    x = synthetic((B, M, K), outliers=True, seed=M + K)
    w = synthetic((B, K, N), std=0.02, seed=K + N)
    qb = get_quant("b200_per_block_2d").fn(w.to(DEV), block_m=128, block_n=128)
    if b_layout == "k":
        qb.tensor = qb.tensor.transpose(1, 2).contiguous().transpose(1, 2)
    out, qx = quant_bmm_fused(x.to(DEV), qb, return_quantized=True, fuse=fuse)
    yx, sx = oracle.per_block_quant(x, block_m=1, block_n=128)
    assert_bytes_equal(qx.tensor, yx, "fused quantized x")
    assert_scales_equal(qx.dequant_scale, sx, "fused x scales")
    ref = oracle.scaled_bmm_promoted_reference(yx, sx, qb.tensor, qb.dequant_scale, qbm=1, qbk=128, qbn=128,
                                               out_dtype=torch.float32)
    assert_bmm_close(out, ref, f"fused={fuse} {shape} {b_layout}")


@pytest.mark.parametrize("fuse", [True, False])
def test_fused_bias_gelu_per_channel_b(fuse):
    B, M, K, N = 1, 192, 384, 320
    x = synthetic((B, M, K), seed=3)
    w = synthetic((B, K, N), std=0.05, seed=4)
    bias = synthetic((B, M, N), seed=5, dtype=torch.float32)
    qb = get_quant("b200_per_channel").fn(w.to(DEV), channel_axis=-1)
    out = quant_bmm_fused(x.to(DEV), qb, bias=bias.to(DEV), activation="gelu", out_dtype=torch.float32, fuse=fuse)
    yx, sx = oracle.per_block_quant(x, block_m=1, block_n=128)
    acc = oracle.scaled_bmm_promoted_reference(
        yx, sx, qb.tensor, qb.dequant_scale.unsqueeze(1).expand(B, (K + 127) // 128, N).contiguous(),
        qbm=1, qbk=128, qbn=1, bias=bias, activation="gelu", out_dtype=torch.float32)
    assert_bmm_close(out, acc, "fused per-channel B")


def test_fused_cfg4_rows_vs_unfused():
    """cfg4 shape slice (rows 0..2047 of [16384,4096] x [4096,14336])."""
    M, K, N = 2048, 4096, 14336
    x = synthetic((M, K), seed=6).to(DEV)
    w = synthetic((K, N), std=0.02, seed=7).to(DEV)
    qb = get_quant("b200_per_block_2d").fn(w.unsqueeze(0), block_m=128, block_n=128)
    out, qx = quant_bmm_fused(x, qb, return_quantized=True, fuse=True)
    qa = get_quant("b200_per_block_2d").fn(x.unsqueeze(0), block_m=1, block_n=128)
    assert torch.equal(qx.tensor.view(torch.uint8), qa.tensor[0].view(torch.uint8))
    ref = torch.bmm(qa.dequantize(), qb.dequantize())[0]
    assert_bmm_close(out, ref, "cfg4 slice")
