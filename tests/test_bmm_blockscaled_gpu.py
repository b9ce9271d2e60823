"""Block-scaled GEMM (power-of-two / E8M0 scales applied by the tensor core,
pcb_bmm_block_scaled) and the E8M0 recipe of the FP8 training linear, against
the fp32 per-128-K-group promotion reference of the oracle."""

import pytest
import torch

import oracle
from practice_cuda_b200.fp8_linear import FP8BlockLinear
from practice_cuda_b200.impls._common import bmm_scaled
from tests._util import assert_bmm_close, synthetic

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _ref(a, sa, qbm, b, sb, qbn):
    return oracle.scaled_bmm_promoted_reference(a, sa, b, sb, qbm=qbm, qbk=128, qbn=qbn, out_dtype=torch.float32)


def _run(a, sa, sa_strides, qbm, b, sb, sb_strides, qbn, out_dtype=torch.bfloat16, bias=None, activation="none"):
    batch, m, _ = a.shape
    out = torch.empty((batch, m, b.shape[-1]), device=DEV, dtype=out_dtype)
    return bmm_scaled(a, b, out, scale_a=sa, sa_strides=sa_strides, qbm=qbm, scale_b=sb, sb_strides=sb_strides,
                      qbn=qbn, qbk=128, bias=bias, activation=activation, block_scaled=True)


@pytest.mark.parametrize("b_layout", ["n", "k"])
@pytest.mark.parametrize("shape", [(2, 300, 640, 264), (1, 1024, 7168, 2048), (3, 128, 128, 136)])
def test_block_scaled_1x128_128x128(shape, b_layout):
    batch, m, k, n = shape
    x = synthetic((batch, m, k), outliers=True, seed=sum(shape))
    w = synthetic((batch, k, n), std=0.02, seed=sum(shape) + 1)
    qa, sa = oracle.per_block_quant_pow2(x, block_m=1, block_n=128)       # sa [B, M, K/128]
    qb, sb = oracle.per_block_quant_pow2(w, block_m=128, block_n=128)     # sb [B, K/128, N/128]
    a_d, sa_d, sb_d = qa.to(DEV), sa.to(DEV), sb.to(DEV)
    b_d = qb.to(DEV) if b_layout == "n" else qb.transpose(1, 2).contiguous().to(DEV).transpose(1, 2)
    out = _run(a_d, sa_d, tuple(sa_d.stride()), 1, b_d, sb_d, tuple(sb_d.stride()), 128)
    assert_bmm_close(out, _ref(qa, sa, 1, qb, sb, 128), f"{shape} B {b_layout}-major")


def test_block_scaled_per_column_b_and_m_major_a():
    """The wgrad shape: A M-major with per-row scales, B N-major with a
    scale per column and K block (128x1 quantization along K of both)."""
    t, o, i = 512, 384, 264
    dy = synthetic((t, o), std=0.1, outliers=True, seed=7)
    x = synthetic((t, i), seed=8)
    qdy, sdy = oracle.per_block_quant_pow2(dy, block_m=128, block_n=1)   # sdy [T/128, O]
    qx, sx = oracle.per_block_quant_pow2(x, block_m=128, block_n=1)      # sx [T/128, I]
    a = qdy.to(DEV).t().unsqueeze(0)                                     # [1, O, T], M-major
    sa = sdy.to(DEV)
    b = qx.to(DEV).unsqueeze(0)                                          # [1, T, I], N-major
    sb = sx.to(DEV)
    out = _run(a, sa, (0, sa.stride(1), sa.stride(0)), 1, b, sb, (0,) + tuple(sb.stride()), 1, torch.float32)
    ref = _ref(qdy.t().unsqueeze(0), sdy.t().unsqueeze(0), 1, qx.unsqueeze(0), sx.unsqueeze(0), 1)
    assert_bmm_close(out, ref, "wgrad layout")


def test_block_scaled_bias_gelu_two_calls():
    x = synthetic((1, 200, 256), seed=11)
    w = synthetic((1, 256, 136), std=0.02, seed=12)
    bias = synthetic((1, 200, 136), seed=13).to(DEV)
    qa, sa = oracle.per_block_quant_pow2(x, block_m=1, block_n=128)
    qb, sb = oracle.per_block_quant_pow2(w, block_m=128, block_n=128)
    ref = torch.nn.functional.gelu(_ref(qa, sa, 1, qb, sb, 128) + bias.float().cpu())
    for _ in range(2):
        out = _run(qa.to(DEV), sa.to(DEV), tuple(sa.stride()), 1, qb.to(DEV), sb.to(DEV), tuple(sb.stride()), 128,
                   bias=bias, activation="gelu")
        assert_bmm_close(out, ref, "bias + gelu")


@pytest.mark.parametrize("t,din,dout", [(256, 384, 512), (384, 256, 128)])
def test_fp8_linear_e8m0_forward_backward(t, din, dout):
    x = synthetic((t, din), outliers=True, seed=1)
    w = synthetic((dout, din), std=0.02, seed=2, dtype=torch.float32)
    dy = synthetic((t, dout), std=0.1, seed=3)
    lin = FP8BlockLinear(din, dout, bias=False).cuda()
    lin.scaling = "e8m0"
    with torch.no_grad():
        lin.weight.copy_(w)
    xg = x.cuda().requires_grad_(True)
    y = lin(xg)
    y.backward(dy.cuda())
    q = oracle.per_block_quant_pow2
    qx, sx = q(x, block_m=1, block_n=128)
    qw, sw = q(w, block_m=128, block_n=128)
    two_d = lambda a, sa, qbm, b, sb, qbn: _ref(a.unsqueeze(0), sa.unsqueeze(0), qbm, b.unsqueeze(0), sb.unsqueeze(0), qbn)[0]
    assert_bmm_close(y.float(), two_d(qx, sx, 1, qw.t(), sw.t(), 128), "forward")
    qdy, sdy = q(dy, block_m=1, block_n=128)
    assert_bmm_close(xg.grad.float(), two_d(qdy, sdy, 1, qw, sw, 128), "dgrad")
    qdyt, sdyt = q(dy, block_m=128, block_n=1)
    qxt, sxt = q(x, block_m=128, block_n=1)
    assert_bmm_close(lin.weight.grad.float(), two_d(qdyt.t(), sdyt.t(), 1, qxt, sxt, 1), "wgrad")


def test_registry_e8m0_scheme_runs_block_scaled():
    """The registry scheme b200_per_block_e8m0_1x128_128x128 quantizes with
    power-of-two scales and its BMM matches the promotion reference."""
    from practice_cuda_b200 import get_bmm, get_quant

    x = synthetic((2, 256, 384), outliers=True, seed=21)
    w = synthetic((2, 384, 264), std=0.02, seed=22)
    impl = get_bmm("b200_per_block_e8m0_1x128_128x128_a_k_b_n")
    quant = get_quant(impl.quant_impl).fn
    qa = quant(x.to(DEV), **impl.quant_a_kwargs)
    qb = quant(w.to(DEV), **impl.quant_b_kwargs)
    assert qa.meta["scale_format"] == "e8m0" and qb.meta["scale_format"] == "e8m0"
    out = impl.fn(qa, qb)
    ref = _ref(qa.tensor.cpu(), qa.dequant_scale.cpu(), 1, qb.tensor.cpu(), qb.dequant_scale.cpu(), 128)
    assert_bmm_close(out, ref, "registry e8m0")
