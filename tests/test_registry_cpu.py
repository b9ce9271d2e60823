"""Host-side logic of the registry and impl wrappers (no GPU): names,
layouts, and the reference's validation errors (raised before any launch)."""

import pytest
import torch

from practice_cuda_b200 import QuantResult, bmm_impl_names, get_bmm, get_quant, registry
from practice_cuda_b200.impls._common import a_layout, matrix_layout

E4M3 = torch.float8_e4m3fn


def test_reference_names_resolve():
    for name in ["triton_per_block_1d", "triton_per_block_2d", "triton_per_channel", "triton_per_tensor",
                 "torch_compile_per_channel", "triton_per_channel_one_pass"]:
        assert get_quant(name).fn is not None
    for q in ["triton_per_block_1d", "triton_per_block_2d", "triton_per_channel", "triton_per_tensor",
              "b200_per_block_1x128_128x128", "b200_per_block_e8m0_1x128_128x128"]:
        for layout in ["a_k_b_k", "a_k_b_n", "a_k_b_n_transpose", "a_m_b_n", "a_m_transpose_b_n_transpose"]:
            impl = get_bmm(f"{q}_{layout}")
            assert impl.quant_impl == q
            assert impl.layout == ("k" if layout.endswith("b_k") else "n")
            assert impl.a_layout == ("m" if layout.startswith("a_m") else "k")


def test_bmm_name_order_groups_by_quant():
    names = bmm_impl_names()
    assert names[0].startswith("b200_per_block_1d")
    assert len(names) == len(set(names)) == 5 * 10  # 9 quant schemes incl. the reference aliases + e8m0


def test_duplicate_registration_rejected():
    with pytest.raises(ValueError, match="duplicate"):
        registry.register_quant("b200_per_tensor", lambda x: x)
    with pytest.raises(ValueError, match="a_layout"):
        registry.register_bmm("x_new", lambda a, b: a, quant_impl="q", layout="n", prepare_b=lambda v: v, a_layout="z")


def test_unknown_names():
    with pytest.raises(KeyError, match="unknown quant"):
        get_quant("nope")
    with pytest.raises(KeyError, match="unknown BMM"):
        get_bmm("nope")


def test_layout_helpers():
    t = torch.zeros(2, 4, 8)
    assert matrix_layout(t, "B") == "n-major"
    assert matrix_layout(t.transpose(1, 2), "B") == "k-major"
    assert a_layout(t) == "k-major" and a_layout(t.transpose(1, 2)) == "m-major"
    with pytest.raises(ValueError, match="contiguous along one matrix dimension"):
        matrix_layout(torch.zeros(4, 4, 4)[:, ::2, ::2], "B")


def test_quant_validation_errors():
    q = get_quant("b200_per_block_2d").fn
    with pytest.raises(ValueError, match="2D or 3D"):
        q(torch.zeros(4))
    with pytest.raises(ValueError, match="power-of-two"):
        q(torch.zeros(4, 4), block_m=3)
    with pytest.raises(ValueError, match="CUDA tensor"):
        q(torch.zeros(4, 4))
    pc = get_quant("b200_per_channel_one_pass").fn
    with pytest.raises(ValueError, match="up to 4096"):
        pc(torch.zeros(2, 5000), channel_axis=-2)
    with pytest.raises(ValueError, match="channel_axis"):
        get_quant("b200_per_channel").fn(torch.zeros(2, 4), channel_axis=0)


def _qr(t, scale, gran, meta):
    return QuantResult(t, scale, "t", gran, meta)


def test_bmm_validation_errors():
    fn = get_bmm("b200_per_block_2d_a_k_b_n").fn
    a = torch.zeros(1, 128, 256).to(E4M3)
    b = torch.zeros(1, 256, 128).to(E4M3)
    qa = _qr(a, torch.ones(1, 1, 2), "block", {"block_m": 128, "block_n": 128})
    qb = _qr(b, torch.ones(1, 2, 1), "block", {"block_m": 128, "block_n": 128})
    with pytest.raises(ValueError, match="3D"):
        fn(_qr(a[0], qa.dequant_scale, "block", qa.meta), qb)
    with pytest.raises(ValueError, match="activation"):
        fn(qa, qb, activation="relu")
    with pytest.raises(ValueError, match="shape mismatch"):
        fn(qa, _qr(torch.zeros(1, 128, 128).to(E4M3), torch.ones(1, 1, 1), "block", qb.meta))
    with pytest.raises(ValueError, match="same K quant block"):
        fn(qa, _qr(b, qb.dequant_scale, "block", {"block_m": 256, "block_n": 128}))
    with pytest.raises(ValueError, match="dequant scale must have shape"):
        fn(qa, _qr(b, torch.ones(1, 3, 1), "block", qb.meta))
    with pytest.raises(ValueError, match="quant_block_k >= 128"):
        fn(_qr(a, torch.ones(1, 2, 4), "block", {"block_m": 64, "block_n": 64}),
           _qr(b, torch.ones(1, 4, 2), "block", {"block_m": 64, "block_n": 64}))
    with pytest.raises(ValueError, match="block granularity"):
        fn(_qr(a, torch.ones(1, 128), "channel", {"channel_axis": -2}), qb)
    with pytest.raises(ValueError, match="out must have shape"):
        fn(qa, qb, out=torch.empty(1, 128, 64, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="do_transpose_b=True requires an N-major"):
        get_bmm("b200_per_block_2d_a_k_b_n").fn(qa, _qr(b.transpose(1, 2).contiguous().transpose(1, 2),
                                                         qb.dequant_scale, "block", qb.meta), do_transpose_b=True)


def test_per_channel_bmm_validation():
    fn = get_bmm("b200_per_channel_a_k_b_n").fn
    a = torch.zeros(1, 16, 32).to(E4M3)
    b = torch.zeros(1, 32, 8).to(E4M3)
    qa = _qr(a, torch.ones(1, 16), "channel", {"channel_axis": -2})
    qb = _qr(b, torch.ones(1, 8), "channel", {"channel_axis": -1})
    with pytest.raises(ValueError, match="channel_axis=-1"):
        fn(qa, _qr(b, torch.ones(1, 8), "channel", {"channel_axis": -2}))
    with pytest.raises(ValueError, match="float32"):
        fn(_qr(a, torch.ones(1, 16, dtype=torch.float64), "channel", {"channel_axis": -2}), qb)


def test_dequantize_semantics_cpu():
    t = torch.tensor([[1.0, 2.0, 3.0], [4.0, 5.0, 6.0]]).to(E4M3)
    q = _qr(t, torch.tensor([[2.0, 3.0]]), "block", {"block_m": 2, "block_n": 2})
    assert torch.equal(q.dequantize(), torch.tensor([[2.0, 4.0, 9.0], [8.0, 10.0, 18.0]]))
    q = _qr(t, torch.tensor([2.0, 3.0]), "channel", {"channel_axis": -2})
    assert torch.equal(q.dequantize(), torch.tensor([[2.0, 4.0, 6.0], [12.0, 15.0, 18.0]]))
    with pytest.raises(ValueError, match="one fewer dimension"):
        _qr(t, torch.ones(2, 1), "channel", {"channel_axis": -1}).dequantize()
