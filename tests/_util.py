"""Shared helpers for the tests: seeded synthetic inputs and tolerances."""

from __future__ import annotations

import torch

E4M3 = torch.float8_e4m3fn
E5M2 = torch.float8_e5m2


def synthetic(shape, *, std=1.0, outliers=False, seed=0, dtype=torch.bfloat16):
    """CPU-generated N(0, std) with numel//1000 entries x100 (BASELINE inputs)."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(shape, generator=g, dtype=torch.float32) * std
    if outliers:
        flat = x.view(-1)
        idx = torch.randperm(flat.numel(), generator=g)[: max(1, flat.numel() // 1000)]
        flat[idx] *= 100.0
    return x.to(dtype)


def u8(t: torch.Tensor) -> torch.Tensor:
    return t.contiguous().view(torch.uint8)


def assert_bytes_equal(actual: torch.Tensor, expected: torch.Tensor, what: str = "") -> None:
    a, e = u8(actual.cpu()), u8(expected.cpu())
    if not torch.equal(a, e):
        bad = (a != e).nonzero()
        raise AssertionError(f"{what}: {bad.shape[0]} bytes differ, first at {bad[0].tolist()}: "
                             f"{a[tuple(bad[0])].item()} vs {e[tuple(bad[0])].item()}")


def assert_scales_equal(actual: torch.Tensor, expected: torch.Tensor, what: str = "") -> None:
    a, e = actual.cpu(), expected.cpu()
    assert a.shape == e.shape, f"{what}: shape {tuple(a.shape)} vs {tuple(e.shape)}"
    if not torch.equal(a.view(torch.int32), e.view(torch.int32)):
        bad = (a.view(torch.int32) != e.view(torch.int32)).nonzero()
        raise AssertionError(f"{what}: {bad.shape[0]} scales differ, first at {bad[0].tolist()}: "
                             f"{a[tuple(bad[0])].item()!r} vs {e[tuple(bad[0])].item()!r}")


# GEMM tolerance (fp32 accumulation order differs from the CPU reference; bf16
# output rounding is 2^-9 relative): elementwise |d| <= RTOL*|ref| + ATOL_FRAC*max|ref|,
# and the max relative error max|d| / max|ref| <= MAX_REL.
RTOL = 1e-2
ATOL_FRAC = 1e-3
MAX_REL = 1e-2


def assert_bmm_close(actual: torch.Tensor, expected: torch.Tensor, what: str = "",
                     rtol: float = RTOL, atol_frac: float = ATOL_FRAC, max_rel: float = MAX_REL) -> float:
    a = actual.float().cpu()
    e = expected.float().cpu()
    assert a.shape == e.shape, f"{what}: shape {tuple(a.shape)} vs {tuple(e.shape)}"
    assert torch.isfinite(a).all(), f"{what}: non-finite output"
    scale = e.abs().max().item()
    d = (a - e).abs()
    rel = d.max().item() / max(scale, 1e-30)
    ok = d <= rtol * e.abs() + atol_frac * scale
    if not bool(ok.all()):
        bad = (~ok).nonzero()[0].tolist()
        raise AssertionError(f"{what}: {int((~ok).sum())} elements out of tolerance, first at {bad}: "
                             f"{a[tuple(bad)].item()} vs {e[tuple(bad)].item()} (max rel {rel:.3e})")
    assert rel <= max_rel, f"{what}: max rel err {rel:.3e} > {max_rel}"
    return rel
