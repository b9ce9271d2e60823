"""The CPU oracle against the golden vectors produced by the reference's own
torch functions (tests/golden/make_golden.py).  Bit-exact for bytes and scales."""

import pytest
import torch

import oracle

E4M3 = torch.float8_e4m3fn


def _u8(t):
    return t.contiguous().view(torch.uint8)


def _cases(golden, kind):
    return sorted(k for k, v in golden.items() if v["kind"] == kind)


def test_golden_has_all_kinds(golden):
    kinds = {v["kind"] for v in golden.values()}
    assert kinds == {"per_channel", "per_block", "per_tensor", "bmm", "legacy_bmm", "float8_dynamic"}


def test_per_channel(golden):
    for name in _cases(golden, "per_channel"):
        c = golden[name]
        y, s = oracle.per_channel_quant(c["x"], channel_axis=c["channel_axis"])
        assert torch.equal(_u8(y), c["y_u8"]), name
        assert torch.equal(s, c["scale"]), name


def test_per_block(golden):
    for name in _cases(golden, "per_block"):
        c = golden[name]
        y, s = oracle.per_block_quant(c["x"], block_m=c["block_m"], block_n=c["block_n"])
        assert torch.equal(_u8(y), c["y_u8"]), name
        assert torch.equal(s, c["scale"]), name


def test_per_tensor_legacy(golden):
    for name in _cases(golden, "per_tensor"):
        c = golden[name]
        dt = torch.float8_e5m2 if "e5m2" in c["fp8_dtype"] else E4M3
        y, r = oracle.legacy_per_tensor_quant(c["x"], quant_dtype=dt, fp8_range=c["fp8_range"])
        assert torch.equal(_u8(y), c["y_u8"]), name
        assert torch.equal(r, c["scale"]), name
        if dt == E4M3:
            y2, r2 = oracle.per_tensor_quant(c["x"])
            assert torch.equal(_u8(y2), c["y_u8"]), name
            assert torch.equal(r2, c["scale"]), name


def test_float8_dynamic_cast(golden):
    """The FP8 training linear's dynamic casts (tensorwise / axiswise, E4M3 /
    E5M2) against the reference's hp_tensor_to_float8_dynamic."""
    names = _cases(golden, "float8_dynamic")
    assert len(names) == 12
    for name in names:
        c = golden[name]
        dt = torch.float8_e5m2 if "e5m2" in c["fp8_dtype"] else E4M3
        y, s = oracle.float8_dynamic_cast(c["x"], dt, axiswise=c["axiswise"])
        assert torch.equal(_u8(y), c["y_u8"]), name
        assert s.shape == c["scale"].shape and torch.equal(s, c["scale"]), name


def _gran(kind):
    if kind[0] == "block":
        return "block", {"block_m": kind[1], "block_n": kind[2]}
    if kind[0] == "channel":
        return "channel", {"channel_axis": kind[1]}
    return "tensor", {}


def test_bmm_dequant_reference(golden):
    for name in _cases(golden, "bmm"):
        c = golden[name]
        a = c["a_u8"].view(E4M3)
        b = c["b_u8"].view(E4M3)
        ag, am = _gran(c["a_kind"])
        bg, bm = _gran(c["b_kind"])
        out = oracle.scaled_bmm_dequant_reference(
            a, c["a_scale"], ag, am, b, c["b_scale"], bg, bm,
            bias=c["bias"], out_dtype=torch.float32)
        assert torch.equal(out, c["out_f32"]), name


def test_bmm_promoted_matches_dequant(golden):
    """The promotion-order reference agrees with the dequant reference to fp32
    rounding (the tolerance the GPU tests build on)."""
    for name in _cases(golden, "bmm"):
        c = golden[name]
        if c["a_kind"][0] != "block":
            continue
        _, qbm, qbk = c["a_kind"]
        _, _, qbn = c["b_kind"]
        out = oracle.scaled_bmm_promoted_reference(
            c["a_u8"].view(E4M3), c["a_scale"], c["b_u8"].view(E4M3), c["b_scale"],
            qbm=qbm, qbk=qbk, qbn=qbn, bias=c["bias"], out_dtype=torch.float32)
        ref = c["out_f32"]
        tol = 1e-5 * ref.abs().max().item()
        assert (out - ref).abs().max().item() <= tol, name


def test_legacy_bmm(golden):
    c = golden["legacy_bmm"]
    out = oracle.legacy_bmm_reference(c["a_u8"].view(E4M3), c["b_u8"].view(E4M3), c["scale"],
                                      bias=c["bias"], out_dtype=torch.float32)
    assert torch.equal(out, c["out_f32"])


@pytest.mark.parametrize("shape", [(4096, 7168)])
def test_oracle_cfg1_scale_shapes(shape):
    """Scale storage shapes at the BASELINE cfg1 activation shape (1x128)."""
    x = torch.zeros(shape, dtype=torch.bfloat16)
    x[0, 0] = 1.0
    y, s = oracle.per_block_quant(x[:128], block_m=1, block_n=128)
    assert s.shape == (128, 56)
    assert y.dtype == E4M3
