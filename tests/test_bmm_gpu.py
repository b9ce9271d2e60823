"""Scaled FP8 BMM (tcgen05 kernel) vs the CPU references.

Tolerance (tests/_util.py): elementwise |C-ref| <= 1e-2*|ref| + 1e-3*max|ref|
and max|C-ref|/max|ref| <= 1e-2, the north-star bar for bf16 output.
"""

import pytest
import torch

import oracle
from practice_cuda_b200 import QuantResult, _lib, get_bmm, get_quant
from tests._util import E4M3, E5M2, assert_bmm_close, synthetic

pytestmark = pytest.mark.gpu

DEV = "cuda"

SCHEMES = {
    # name: (quant impl, A block, B block)
    "1x128_128x128": ("b200_per_block_1x128_128x128", (1, 128), (128, 128)),
    "1d": ("b200_per_block_1d", (1, 128), (128, 1)),
    "2d": ("b200_per_block_2d", (128, 128), (128, 128)),
}
LAYOUTS = ["a_k_b_k", "a_k_b_n", "a_k_b_n_transpose", "a_m_b_n", "a_m_transpose_b_n_transpose"]


def _relayout(q: QuantResult, *, mn_major: bool) -> QuantResult:
    """Same values, storage contiguous along dim -2 (mn_major) or dim -1."""
    t = q.tensor
    if mn_major:
        t = t.transpose(-1, -2).contiguous().transpose(-1, -2)
    else:
        t = t.contiguous()
    return QuantResult(t, q.dequant_scale, q.impl, q.granularity, dict(q.meta))


def _operands_for_layout(qa, qb, layout):
    a_m = layout.startswith("a_m")
    b_k = layout.endswith("b_k")
    qa = _relayout(qa, mn_major=a_m)
    qb = _relayout(qb, mn_major=b_k)
    return qa, qb


def _quant_pair(scheme, a, b):
    qname, ablk, bblk = SCHEMES[scheme]
    qf = get_quant(qname).fn
    qa = qf(a.to(DEV), block_m=ablk[0], block_n=ablk[1])
    qb = qf(b.to(DEV), block_m=bblk[0], block_n=bblk[1])
    return qa, qb, ablk, bblk


def _promoted_ref(qa, qb, ablk, bblk, bias=None, activation="none"):
    return oracle.scaled_bmm_promoted_reference(
        qa.tensor, qa.dequant_scale, qb.tensor, qb.dequant_scale,
        qbm=ablk[0], qbk=ablk[1], qbn=bblk[1], bias=bias, activation=activation, out_dtype=torch.float32)


@pytest.mark.parametrize("scheme", list(SCHEMES))
@pytest.mark.parametrize("layout", LAYOUTS)
@pytest.mark.parametrize("shape", [(2, 128, 256, 128), (1, 200, 384, 136), (3, 64, 200, 300)])
def test_per_block_layouts(scheme, layout, shape):
    B, M, K, N = shape
    a = synthetic((B, M, K), outliers=True, seed=M + K)
    b = synthetic((B, K, N), std=0.02, seed=K + N)
    qa, qb, ablk, bblk = _quant_pair(scheme, a, b)
    ref = _promoted_ref(qa, qb, ablk, bblk)
    qa2, qb2 = _operands_for_layout(qa, qb, layout)
    impl = get_bmm(f"{SCHEMES[scheme][0]}_{layout}")
    qa2, qb2 = impl.prepare_a(qa2), impl.prepare_b(qb2)
    out = impl.fn(qa2, qb2, out_dtype=torch.bfloat16)
    assert out.shape == (B, M, N) and out.dtype == torch.bfloat16
    assert_bmm_close(out, ref, f"{scheme} {layout} {shape}")


def test_golden_bmm(golden):
    for name, c in golden.items():
        if c["kind"] != "bmm":
            continue
        def qr(prefix, kind):
            t = c[f"{prefix}_u8"].view(E4M3).to(DEV)
            s = c[f"{prefix}_scale"].to(DEV)
            if kind[0] == "block":
                return QuantResult(t, s, "golden", "block", {"block_m": kind[1], "block_n": kind[2]})
            if kind[0] == "channel":
                return QuantResult(t, s, "golden", "channel", {"channel_axis": kind[1]})
            return QuantResult(t, s, "golden", "tensor", {})
        qa, qb = qr("a", c["a_kind"]), qr("b", c["b_kind"])
        bias = c["bias"].to(DEV) if c["bias"] is not None else None
        if c["a_kind"][0] == "block":
            fn = get_bmm("b200_per_block_2d_a_k_b_n").fn
        elif c["a_kind"][0] == "channel":
            fn = get_bmm("b200_per_channel_a_k_b_n").fn
        else:
            fn = get_bmm("b200_per_tensor_a_k_b_n").fn
        out = fn(qa, qb, out_dtype=torch.float32, bias=bias)
        assert_bmm_close(out, c["out_f32"], name)


@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("activation", ["none", "gelu"])
def test_bias_activation_out_dtype(out_dtype, activation):
    B, M, K, N = 2, 130, 256, 260
    a = synthetic((B, M, K), seed=1)
    b = synthetic((B, K, N), std=0.05, seed=2)
    bias = synthetic((B, M, N), seed=3, dtype=torch.float32)
    qa, qb, ablk, bblk = _quant_pair("1x128_128x128", a, b)
    ref = _promoted_ref(qa, qb, ablk, bblk, bias=bias, activation=activation)
    out = get_bmm("b200_per_block_1x128_128x128_a_k_b_n").fn(
        qa, qb, out_dtype=out_dtype, bias=bias.to(DEV), activation=activation)
    assert out.dtype == out_dtype
    assert_bmm_close(out, ref, f"{out_dtype} {activation}")


@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("shape", [(2, 300, 384, 264), (1, 260, 256, 520), (3, 384, 128, 136)])
def test_pair_tma_store_ragged(out_dtype, shape):
    """CTA-pair tiles whose bf16 / fp16 / fp32 output rows are 16-byte aligned leave
    through TMA box stores; rows and columns past M and N (partial 256 x 256
    tiles, partial 32 x 64 boxes) must be clipped, with bias and GELU applied."""
    B, M, K, N = shape
    a = synthetic((B, M, K), outliers=True, seed=M + 1)
    b = synthetic((B, K, N), std=0.05, seed=N + 2)
    bias = synthetic((B, M, N), seed=3, dtype=torch.float32)
    qa, qb, ablk, bblk = _quant_pair("1x128_128x128", a, b)
    ref = _promoted_ref(qa, qb, ablk, bblk, bias=bias, activation="gelu")
    out = torch.full((B, M, N), float("nan"), device=DEV, dtype=out_dtype)
    get_bmm("b200_per_block_1x128_128x128_a_k_b_n").fn(qa, qb, out=out, out_dtype=out_dtype, bias=bias.to(DEV),
                                                         activation="gelu")
    assert torch.isfinite(out.float()).all(), "an output element was not written"
    assert_bmm_close(out, ref, f"pair tma store {out_dtype} {shape}")


def test_out_argument_and_k_tail():
    B, M, K, N = 1, 256, 200, 256  # K = 128 + 72: a partial second K group
    a = synthetic((B, M, K), seed=4)
    b = synthetic((B, K, N), std=0.02, seed=5)
    qa, qb, ablk, bblk = _quant_pair("2d", a, b)
    out = torch.empty((B, M, N), device=DEV, dtype=torch.bfloat16)
    res = get_bmm("b200_per_block_2d_a_k_b_n").fn(qa, qb, out=out)
    assert res.data_ptr() == out.data_ptr()
    assert_bmm_close(out, _promoted_ref(qa, qb, ablk, bblk), "k tail")


@pytest.mark.parametrize("layout", LAYOUTS)
@pytest.mark.parametrize("shape", [(1, 256, 512, 256), (3, 33, 47, 65), (2, 100, 4096, 72)])
def test_per_channel(layout, shape):
    B, M, K, N = shape
    a = synthetic((B, M, K), seed=6)
    b = synthetic((B, K, N), std=0.02, seed=7)
    qf = get_quant("b200_per_channel").fn
    qa = qf(a.to(DEV), channel_axis=-2)
    qb = qf(b.to(DEV), channel_axis=-1)
    ref = oracle.scaled_bmm_dequant_reference(qa.tensor, qa.dequant_scale, "channel", {"channel_axis": -2},
                                              qb.tensor, qb.dequant_scale, "channel", {"channel_axis": -1},
                                              out_dtype=torch.float32)
    qa2, qb2 = _operands_for_layout(qa, qb, layout)
    out = get_bmm(f"b200_per_channel_{layout}").fn(qa2, qb2)
    assert_bmm_close(out, ref, f"channel {layout} {shape}")


@pytest.mark.parametrize("layout", ["a_k_b_n", "a_k_b_k", "a_m_b_n"])
def test_per_tensor(layout):
    B, M, K, N = 2, 192, 320, 160
    a = synthetic((B, M, K), seed=8)
    b = synthetic((B, K, N), std=0.02, seed=9)
    qf = get_quant("b200_per_tensor").fn
    qa, qb = qf(a.to(DEV)), qf(b.to(DEV))
    ref = oracle.scaled_bmm_dequant_reference(qa.tensor, qa.dequant_scale, "tensor", {},
                                              qb.tensor, qb.dequant_scale, "tensor", {}, out_dtype=torch.float32)
    qa2, qb2 = _operands_for_layout(qa, qb, layout)
    out = get_bmm(f"b200_per_tensor_{layout}").fn(qa2, qb2)
    assert_bmm_close(out, ref, f"tensor {layout}")
    combined = (qa.dequant_scale * qb.dequant_scale).reshape(1)
    out2 = get_bmm(f"b200_per_tensor_{layout}").fn(qa2, qb2, dequant_scale=combined)
    assert torch.equal(out.cpu(), out2.cpu())


def test_e5m2_operands():
    B, M, K, N = 1, 128, 256, 128
    a = synthetic((B, M, K), seed=10)
    b = synthetic((B, K, N), std=0.02, seed=11)
    qf = get_quant("b200_per_block_2d").fn
    qa = qf(a.to(DEV), block_m=1, block_n=128, fp8_dtype=E5M2)
    qb = qf(b.to(DEV), block_m=128, block_n=128, fp8_dtype=E5M2)
    ref = _promoted_ref(qa, qb, (1, 128), (128, 128))
    out = get_bmm("b200_per_block_1x128_128x128_a_k_b_n").fn(qa, qb)
    assert_bmm_close(out, ref, "e5m2")


def _gpu_fp32_reference(qa, qb, ablk, bblk):
    """fp32 dequantize-and-matmul on the GPU (torch, TF32 off) for full sizes."""
    assert not torch.backends.cuda.matmul.allow_tf32
    return torch.bmm(qa.dequantize(), qb.dequantize())


def test_cfg3_full_size_sampled_batches():
    """BASELINE cfg3 (B=32, M=4096, K=7168, N=2048, 1x128 / 128x128) at full
    size; batches 0, 17 and 31 checked against an fp32 GPU reference."""
    B, M, K, N = 32, 4096, 7168, 2048
    g = torch.Generator(device=DEV).manual_seed(0)
    a = torch.randn((B, M, K), device=DEV, generator=g)
    flat = a.view(-1)
    idx = torch.randint(0, flat.numel(), (flat.numel() // 1000,), device=DEV, generator=g)
    flat[idx] *= 100
    a = a.bfloat16()
    b = (torch.randn((B, K, N), device=DEV, generator=g) * 0.02).bfloat16()
    qf = get_quant("b200_per_block_1x128_128x128").fn
    qa = qf(a, block_m=1, block_n=128)
    qb = qf(b, block_m=128, block_n=128)
    del a, b
    out = get_bmm("b200_per_block_1x128_128x128_a_k_b_n").fn(qa, qb)
    for bi in (0, 17, 31):
        sa = QuantResult(qa.tensor[bi:bi + 1], qa.dequant_scale[bi:bi + 1], "t", "block", dict(qa.meta))
        sb = QuantResult(qb.tensor[bi:bi + 1], qb.dequant_scale[bi:bi + 1], "t", "block", dict(qb.meta))
        ref = _gpu_fp32_reference(sa, sb, (1, 128), (128, 128))
        assert_bmm_close(out[bi:bi + 1], ref, f"cfg3 batch {bi}")


def test_cfg2_full_size_per_channel():
    M, K, N = 8192, 4096, 4096
    a = synthetic((M, K), seed=20).to(DEV)
    b = synthetic((K, N), std=0.02, seed=21).to(DEV)
    qf = get_quant("b200_per_channel").fn
    qa = qf(a.unsqueeze(0), channel_axis=-2)
    qb = qf(b.unsqueeze(0), channel_axis=-1)
    out = get_bmm("b200_per_channel_a_k_b_n").fn(qa, qb)
    ref = torch.bmm(qa.dequantize(), qb.dequantize())
    assert_bmm_close(out, ref, "cfg2")


def test_injected_error_reported_without_fault():
    """The debug hook makes the kernel write the device error word; the
    context stays usable and the next launch is clean."""
    _lib.device_error()  # clear
    a = synthetic((1, 128, 128), seed=30)
    b = synthetic((1, 128, 128), std=0.02, seed=31)
    qa, qb, ablk, bblk = _quant_pair("2d", a, b)
    _lib.check(_lib.lib().pcb_debug_inject_error(_lib.PCB_ERR_TIMEOUT), "inject")
    out = get_bmm("b200_per_block_2d_a_k_b_n").fn(qa, qb)
    code, site, info = _lib.device_error()
    assert code == _lib.PCB_ERR_TIMEOUT and site == 4
    assert_bmm_close(out, _promoted_ref(qa, qb, ablk, bblk), "after injection")
    out = get_bmm("b200_per_block_2d_a_k_b_n").fn(qa, qb)
    assert _lib.device_error() == (0, 0, 0)


def test_zero_k_and_empty():
    a = torch.empty((2, 64, 0), device=DEV, dtype=E4M3)
    b = torch.empty((2, 0, 32), device=DEV, dtype=E4M3)
    qa = QuantResult(a, torch.ones((2, 64), device=DEV), "t", "channel", {"channel_axis": -2})
    qb = QuantResult(b, torch.ones((2, 32), device=DEV), "t", "channel", {"channel_axis": -1})
    bias = torch.randn((2, 64, 32), device=DEV)
    out = get_bmm("b200_per_channel_a_k_b_n").fn(qa, qb, bias=bias, out_dtype=torch.float32)
    assert torch.equal(out, bias)


@pytest.mark.parametrize("layout", ["a_k_b_n", "a_k_b_k", "a_m_b_n"])
@pytest.mark.parametrize("m", [128, 384])
def test_per_block_pair_and_single(layout, m):
    """Per-block scales on both tile paths: M > 128 runs 256x256 tiles on a
    CTA pair (M = 384 leaves the second CTA of the last pair idle), M <= 128
    runs 128x256 tiles on one CTA."""
    B, M, K, N = 2, m, 640, 512
    a = synthetic((B, M, K), outliers=True, seed=40)
    b = synthetic((B, K, N), std=0.02, seed=41)
    qa, qb, ablk, bblk = _quant_pair("1x128_128x128", a, b)
    ref = _promoted_ref(qa, qb, ablk, bblk)
    qa2, qb2 = _operands_for_layout(qa, qb, layout)
    out = get_bmm(f"b200_per_block_1x128_128x128_{layout}").fn(qa2, qb2)
    assert_bmm_close(out, ref, f"per-block M={m} {layout}")


@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("shape", [(384, 512, 512), (300, 640, 520), (512, 384, 1024)])
def test_per_column_scales_wgrad_layout(out_dtype, shape):
    """The weight-gradient GEMM of the FP8 training linear: A M-major with
    row scales contiguous along M per K group, B N-major with per-column
    scales contiguous along N per K group (16-byte scale loads on full tiles,
    scalar loads on partial ones), fp32 or bf16 output."""
    from practice_cuda_b200.fp8_linear import _gemm

    M, K, N = shape
    g = torch.Generator().manual_seed(M + N)
    a = (torch.randn(M, K, generator=g) * 0.2).to(torch.float8_e4m3fn)
    b = (torch.randn(K, N, generator=g) * 0.2).to(torch.float8_e4m3fn)
    sa_t = torch.rand(K // 128 + (K % 128 > 0), M, generator=g) + 0.5   # [kg, m]
    sb = torch.rand(K // 128 + (K % 128 > 0), N, generator=g) + 0.5     # [kg, n]
    a_dev = a.to(DEV).t().contiguous().t()                             # M-major
    sa_dev, sb_dev = sa_t.to(DEV), sb.to(DEV)
    out = _gemm(a_dev, sa_dev, (sa_dev.stride(1), sa_dev.stride(0)), 1, b.to(DEV), sb_dev, tuple(sb_dev.stride()), 1,
                out_dtype)
    ref = torch.zeros(M, N)
    for kg in range(sa_t.shape[0]):
        ks = slice(128 * kg, min(K, 128 * kg + 128))
        ref += (a[:, ks].float() @ b[ks].float()) * sa_t[kg][:, None] * sb[kg][None, :]
    assert out.dtype == out_dtype
    assert_bmm_close(out, ref, f"wgrad layout {out_dtype} {shape}")
