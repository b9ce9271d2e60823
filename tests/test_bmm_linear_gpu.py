"""The batched FP8 training linear (Float8BMMLinear drop-in) on the GPU.

Casts: bytes and quant scales bit-exact against the oracle's restatement of
``hp_tensor_to_float8_dynamic`` (pinned to the reference by golden vectors).
GEMMs: forward, dgrad and wgrad against the oracle casts dequantized and
multiplied in fp32 on the CPU, with the reference backward's scale folding
for axiswise scaling -- max rel err <= 1e-2 (tests/_util.py).
"""

import pytest
import torch

import oracle
from practice_cuda_b200.bmm_linear import (
    BMMLinear,
    Float8BMMLinear,
    Float8BMMLinearConfig,
    bmm_linear_tma,
    cast_to_float8,
    convert_to_float8_bmm_training,
)
from tests._util import E4M3, E5M2, assert_bmm_close, assert_bytes_equal, assert_scales_equal, synthetic

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.mark.parametrize("axiswise", [False, True])
@pytest.mark.parametrize("dtype", [E4M3, E5M2])
@pytest.mark.parametrize("xdtype", [torch.bfloat16, torch.float32])
def test_cast_matches_oracle(axiswise, dtype, xdtype):
    x = synthetic((3, 50, 272), outliers=True, seed=1, dtype=xdtype)
    x[1, 7] = 0  # a zero row hits the eps clamp
    y, s = cast_to_float8(x.to(DEV), dtype, axiswise)
    y_ref, s_ref = oracle.float8_dynamic_cast(x, dtype, axiswise=axiswise)
    assert_bytes_equal(y, y_ref, "cast bytes")
    assert_scales_equal(s, s_ref, "cast scale")


def _deq(data, scale):
    return data.float() / scale.float()


def _ref_grads(x, w, bias, dy, axis):
    """Forward and both gradients from the oracle's casts, fp32 on the CPU,
    in the order of the reference's _Float8BMMLinearFunction."""
    xd, xs = oracle.float8_dynamic_cast(x, E4M3, axiswise=axis)
    wd, ws = oracle.float8_dynamic_cast(w, E4M3, axiswise=axis)
    y = torch.bmm(_deq(xd, xs), _deq(wd, ws).transpose(-2, -1))
    if bias is not None:
        y = y + bias.float().unsqueeze(1)
    if axis:
        b, n = w.shape[0], w.shape[1]
        m = x.shape[1]
        dyd, dys = oracle.float8_dynamic_cast(dy.float() / ws.reshape(b, n).unsqueeze(1), E5M2, axiswise=True)
        dx = torch.bmm(_deq(dyd, dys), wd.float())
        dytd, dyts = oracle.float8_dynamic_cast(dy.transpose(-2, -1).float() / xs.reshape(b, m).unsqueeze(1), E5M2,
                                                axiswise=True)
        dw = torch.bmm(_deq(dytd, dyts), xd.float())
    else:
        dyd, dys = oracle.float8_dynamic_cast(dy, E5M2, axiswise=False)
        dx = torch.bmm(_deq(dyd, dys), _deq(wd, ws))
        dw = torch.bmm(_deq(dyd, dys).transpose(-2, -1), _deq(xd, xs))
    return y, dx, dw


@pytest.mark.parametrize("granularity", ["tensorwise", "axiswise"])
@pytest.mark.parametrize("bias", [False, True])
def test_forward_dgrad_wgrad(granularity, bias):
    B, M, K, N = 2, 256, 384, 512
    torch.manual_seed(0)
    mod = Float8BMMLinear(B, K, N, bias=bias, config=Float8BMMLinearConfig(scaling_granularity=granularity),
                          device=DEV, dtype=torch.bfloat16)
    x = synthetic((B, M, K), outliers=True, seed=3).to(DEV).requires_grad_(True)
    y = mod(x)
    dy = synthetic((B, M, N), std=0.1, seed=4)
    y.backward(dy.to(DEV))
    torch.cuda.synchronize()
    axis = granularity == "axiswise"
    y_ref, dx_ref, dw_ref = _ref_grads(x.detach().cpu(), mod.weight.detach().cpu(),
                                       mod.bias.detach().cpu() if bias else None, dy, axis)
    assert y.dtype == torch.bfloat16 and y.shape == (B, M, N)
    assert_bmm_close(y, y_ref, f"{granularity} forward")
    assert_bmm_close(x.grad, dx_ref, f"{granularity} dgrad")
    assert_bmm_close(mod.weight.grad, dw_ref, f"{granularity} wgrad")
    if bias:
        torch.testing.assert_close(mod.bias.grad.float().cpu(), dy.float().sum(dim=1), rtol=2e-2, atol=2e-2)


def test_op_semantics_and_fake():
    """``(A @ B) / (sa * sb) + bias`` with quant scales, per-channel and
    tensorwise, mixed E5M2 x E4M3 operands; and the op traces under FakeTensor."""
    B, M, K, N = 2, 128, 256, 192
    a = synthetic((B, M, K), seed=5).to(DEV)
    b = synthetic((B, K, N), std=0.05, seed=6).to(DEV)
    ad, as_ = cast_to_float8(a, E5M2, True)
    bt_d, bs = cast_to_float8(b.transpose(-2, -1).contiguous(), E4M3, True)  # per output column
    bd = bt_d.transpose(-2, -1)
    bias = synthetic((B, N), seed=7).to(DEV)
    out = bmm_linear_tma(ad, bd, as_, bs, bias, True, torch.float32, True)
    ref = (torch.bmm(ad.float().cpu(), bd.float().cpu()) / (as_.cpu() * bs.cpu().transpose(-2, -1))
           + bias.cpu().unsqueeze(1))
    assert_bmm_close(out, ref, "per-channel op")
    ad2, as2 = cast_to_float8(a, E4M3, False)
    bd2, bs2 = cast_to_float8(b, E4M3, False)
    out2 = bmm_linear_tma(ad2, bd2, as2, bs2, ad2, False, torch.bfloat16, False)
    ref2 = torch.bmm(ad2.float().cpu(), bd2.float().cpu()) / (as2.cpu() * bs2.cpu())
    assert_bmm_close(out2, ref2, "tensorwise op")
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode() as mode:
        fa = mode.from_tensor(ad2)
        fb = mode.from_tensor(bd2)
        fs = mode.from_tensor(as2)
        o = torch.ops.pcb200.bmm_linear_tma(fa, fb, fs, fs, fa, False, torch.bfloat16, False)
        assert o.shape == (B, M, N) and o.dtype == torch.bfloat16


def test_convert_and_errors():
    torch.manual_seed(0)
    model = torch.nn.Sequential(BMMLinear(2, 128, 256, device=DEV), torch.nn.ReLU(), BMMLinear(2, 256, 64, device=DEV))
    w0 = model[0].weight
    convert_to_float8_bmm_training(model, Float8BMMLinearConfig(scaling_granularity="axiswise"))
    assert isinstance(model[0], Float8BMMLinear) and isinstance(model[2], Float8BMMLinear)
    assert model[0].weight is w0  # parameters are shared, not copied
    x = torch.randn(2, 32, 128, device=DEV)
    model(x).sum().backward()
    assert model[0].weight.grad is not None and torch.isfinite(model[0].weight.grad).all()
    with pytest.raises(ValueError, match="expects \\[B,M,K\\]"):
        model[0](torch.randn(32, 128, device=DEV))
    with pytest.raises(ValueError, match="input shape mismatch"):
        model[0](torch.randn(2, 32, 100, device=DEV))
    with pytest.raises(ValueError, match="does not support scaling"):
        Float8BMMLinearConfig(scaling_granularity="blockwise")
