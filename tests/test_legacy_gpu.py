"""Ports of the reference's known-answer tests for the legacy entry points
(kernels/fp8_bmm/test/fp8_quant_test.py and fp8_quant_bmm_test.py), run
against the libpcb200-backed shims with the reference's own tolerances."""

import pytest
import torch

import oracle
from practice_cuda_b200 import _lib
from practice_cuda_b200.fp8_warper import FP8Format, fp8_bmm_quant_triton, fp8_quant_triton
from practice_cuda_b200.impls._common import bmm_scaled

pytestmark = pytest.mark.gpu

QUANT_SHAPES = [(128, 256), (17, 33), (32, 2048, 960), (80, 2048, 640), (14, 2048, 8192)]
BMM_SHAPES = [(1, 128, 128, 128), (2, 64, 64, 64), (3, 33, 47, 65), (4, 256, 512, 256)]


@pytest.fixture(autouse=True)
def _seed():
    torch.manual_seed(0)


def _ref(x, **kw):
    y, r = oracle.legacy_per_tensor_quant(x.cpu(), **kw)
    return y, r


# ---------------- fp8_quant_test.py -------------------------------------------
def test_output_dtype():
    for shape in [(128, 256), (4, 64, 128)]:
        out, _ = fp8_quant_triton(torch.randn(shape, device="cuda"))
        assert out.dtype == torch.float8_e4m3fn


@pytest.mark.parametrize("shape", QUANT_SHAPES)
def test_matches_reference(shape):
    x = torch.randn(shape, device="cuda")
    ref, _ = _ref(x)
    out, _ = fp8_quant_triton(x)
    assert out.shape == ref.shape
    assert torch.equal(out.cpu().float(), ref.float())


@pytest.mark.parametrize("shape", QUANT_SHAPES)
def test_reciprocal_factor(shape):
    x = torch.randn(shape, device="cuda")
    _, ref_recip = _ref(x)
    _, recip = fp8_quant_triton(x)
    expected = x.abs().amax().clamp(min=1e-12) / 448.0
    assert torch.allclose(recip, expected, rtol=1e-5, atol=1e-7)
    assert torch.equal(recip.cpu(), ref_recip)


@pytest.mark.parametrize("shape", QUANT_SHAPES)
def test_dequant_roundtrip(shape):
    x = torch.randn(shape, device="cuda")
    out, recip = fp8_quant_triton(x)
    x_hat = out.float() * recip
    assert torch.allclose(x_hat, x, rtol=1e-1, atol=0.05 * x.abs().amax().item())


@pytest.mark.parametrize("shape", QUANT_SHAPES)
def test_output_range(shape):
    out, _ = fp8_quant_triton(torch.randn(shape, device="cuda") * 1000.0)
    assert out.float().abs().amax().item() <= 448.0 + 1e-3


def test_clamping_with_outliers():
    x = torch.randn((64, 64), device="cuda")
    x[0, 0] = 1e6
    x[1, 1] = -1e6
    out, _ = fp8_quant_triton(x)
    o = out.float()
    assert o.abs().amax().item() <= 448.0 + 1e-3
    assert o[0, 0].item() == pytest.approx(448.0, abs=1e-2)
    assert o[1, 1].item() == pytest.approx(-448.0, abs=1e-2)


def test_all_zeros():
    out, recip = fp8_quant_triton(torch.zeros((32, 64), device="cuda"))
    assert not torch.isnan(out.float()).any()
    assert out.float().abs().amax().item() == 0.0
    assert torch.isfinite(recip).item()


def test_e5m2_format():
    x = torch.randn((64, 128), device="cuda")
    ref, _ = _ref(x, quant_dtype=torch.float8_e5m2, fp8_range=57344.0)
    out, _ = fp8_quant_triton(x, quant_dtype=FP8Format.E5M2, fp8_range=FP8Format.E5M2.value.max_fwd)
    assert out.dtype == torch.float8_e5m2
    assert torch.equal(out.cpu().float(), ref.float())


def test_determinism():
    x = torch.randn((64, 128), device="cuda")
    assert torch.equal(fp8_quant_triton(x)[0].float(), fp8_quant_triton(x)[0].float())


def test_bf16_input_scale_in_bf16():
    """The legacy path does its scale arithmetic in x's dtype (bf16 here)."""
    x = torch.randn((96, 200), device="cuda").bfloat16()
    ref, ref_recip = _ref(x)
    out, recip = fp8_quant_triton(x)
    assert recip.dtype == torch.bfloat16
    assert torch.equal(recip.cpu(), ref_recip)
    assert torch.equal(out.cpu().view(torch.uint8), ref.view(torch.uint8))


# ---------------- fp8_quant_bmm_test.py ---------------------------------------
def _rand_fp8(shape, dtype=torch.float8_e4m3fn):
    return (torch.randn(shape, device="cuda") * 0.5).to(dtype)


def _launch(a, b, quant_scale, bias=None, out_dtype=torch.bfloat16):
    """The reference test's launcher (a 2D bias broadcasts over the batch)."""
    B, M, K = a.shape
    if bias is not None and bias.dim() == 2:
        bias = bias.unsqueeze(0).expand(B, -1, -1).contiguous()
    return fp8_bmm_quant_triton(a, b, bias, quant_scale=torch.tensor(float(quant_scale), device="cuda"),
                                out_dtype=out_dtype)


def test_bmm_output_dtypes():
    a, b = _rand_fp8((1, 64, 64)), _rand_fp8((1, 64, 64))
    assert _launch(a, b, 1.0).dtype == torch.bfloat16
    assert _launch(a, b, 1.0, out_dtype=torch.float8_e4m3fn).dtype == torch.float8_e4m3fn


@pytest.mark.parametrize("shape", BMM_SHAPES)
def test_bmm_matches_reference(shape):
    B, M, K, N = shape
    a, b = _rand_fp8((B, M, K)), _rand_fp8((B, K, N))
    ref = oracle.legacy_bmm_reference(a, b, 1.0, out_dtype=torch.bfloat16)
    out = _launch(a, b, 1.0)
    assert out.shape == ref.shape == (B, M, N)
    assert torch.allclose(out.float().cpu(), ref.float(), rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("shape", BMM_SHAPES)
def test_bmm_matches_reference_fp8_out(shape):
    B, M, K, N = shape
    a, b = _rand_fp8((B, M, K)), _rand_fp8((B, K, N))
    ref = oracle.legacy_bmm_reference(a, b, 1.0, out_dtype=torch.float32).clamp(-448, 448).to(torch.float8_e4m3fn)
    out = _launch(a, b, 1.0, out_dtype=torch.float8_e4m3fn)
    assert torch.allclose(out.float().cpu(), ref.float(), rtol=2e-1, atol=1e-1)


@pytest.mark.parametrize("shape", BMM_SHAPES)
def test_bmm_with_bias(shape):
    B, M, K, N = shape
    a, b = _rand_fp8((B, M, K)), _rand_fp8((B, K, N))
    bias = torch.randn((B, M, N), device="cuda")
    ref = oracle.legacy_bmm_reference(a, b, 1.0, bias=bias, out_dtype=torch.bfloat16)
    out = _launch(a, b, 1.0, bias=bias)
    assert torch.allclose(out.float().cpu(), ref.float(), rtol=1e-2, atol=1e-2)


def test_bmm_with_2d_bias_broadcast():
    B, M, K, N = 4, 64, 64, 64
    a, b = _rand_fp8((B, M, K)), _rand_fp8((B, K, N))
    bias = torch.randn((M, N), device="cuda")
    ref = oracle.legacy_bmm_reference(a, b, 1.0, bias=bias, out_dtype=torch.bfloat16)
    out = _launch(a, b, 1.0, bias=bias)
    assert torch.allclose(out.float().cpu(), ref.float(), rtol=1e-2, atol=1e-2)


def test_bmm_quant_scale_applied():
    a, b = _rand_fp8((1, 64, 64)), _rand_fp8((1, 64, 64))
    s1 = _launch(a, b, 1.0, out_dtype=torch.float32)
    s2 = _launch(a, b, 2.0, out_dtype=torch.float32)
    nz = s1.abs() > 1e-3
    ratio = s2[nz] / s1[nz]
    assert torch.allclose(ratio, torch.full_like(ratio, 2.0), rtol=1e-2, atol=1e-2)


def test_bmm_output_range_clamped():
    a, b = _rand_fp8((1, 64, 128)), _rand_fp8((1, 128, 64))
    out = _launch(a, b, 100.0, out_dtype=torch.float8_e4m3fn)
    assert out.float().abs().amax().item() <= 448.0 + 1e-3


def test_bmm_all_zeros():
    a = torch.zeros((2, 32, 64), device="cuda", dtype=torch.float8_e4m3fn)
    b = torch.zeros((2, 64, 32), device="cuda", dtype=torch.float8_e4m3fn)
    out = _launch(a, b, 1.0, out_dtype=torch.float32)
    assert not torch.isnan(out).any()
    assert out.abs().amax().item() == 0.0


def test_bmm_batch_independence():
    B, M, K, N = 2, 32, 32, 32
    a, b = _rand_fp8((B, M, K)), _rand_fp8((B, K, N))
    out = _launch(a, b, 1.0, out_dtype=torch.float32)
    for i in range(B):
        single = _launch(a[i:i + 1], b[i:i + 1], 1.0, out_dtype=torch.float32)
        assert torch.allclose(out[i], single[0], rtol=1e-3, atol=1e-3)


def test_bmm_determinism():
    a, b = _rand_fp8((2, 64, 64)), _rand_fp8((2, 64, 64))
    assert torch.equal(_launch(a, b, 1.0).float(), _launch(a, b, 1.0).float())


def test_microbench_fixed_tile():
    """profile_fixed_b_n.py:277-283: one 64x64x128 tile vs (a@b)*scale in bf16, 2e-2."""
    a = _rand_fp8((1, 64, 128))
    b = _rand_fp8((1, 128, 64))
    scale = 0.5
    out = _launch(a, b, scale)
    ref = ((a.float() @ b.float()) * scale).bfloat16()
    torch.testing.assert_close(out, ref, rtol=2e-2, atol=2e-2)
