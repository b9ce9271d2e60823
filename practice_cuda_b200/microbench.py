"""Fixed-shape FP8 BMM layout variants (the reference's ``--variant`` microbench).

    python -m practice_cuda_b200.microbench --variant {a_k_b_k,a_k_b_k_tma,a_k_b_n,a_k_b_n_tma,a_m_b_n,a_m_b_n_tma}
                                            [--warmup W]

Counterpart of ``fp8_training/microbench/profile_fixed_b_n.py:229-287``: one
M=64, N=64, K=128 FP8 e4m3 GEMM ``C = (A @ B) * scale`` (bf16 out, one fp32
scale) with A K-major or M-major and B K-major or N-major, launched once after
``--warmup`` launches -- a compact single-kernel target for ncu -- and checked
against ``(A.float() @ B.float()) * scale`` rounded to bf16 with rtol = atol =
2e-2, the reference's bar.  The kernel is libpcb200's scaled BMM, which always
stages operands with TMA, so each ``*_tma`` variant runs the same kernel as
its plain counterpart (kept so the reference's command lines work unchanged).
"""

from __future__ import annotations

import argparse

import torch

from .impls._common import bmm_scaled

M, N, K = 64, 64, 128
VARIANTS = ("a_k_b_k", "a_k_b_k_tma", "a_k_b_n", "a_k_b_n_tma", "a_m_b_n", "a_m_b_n_tma")


def make_operands(variant: str, device="cuda"):
    """The reference's operands for ``variant`` (seed 0, N(0, 0.25^2) in bf16
    cast to e4m3, the layouts of profile_fixed_b_n.py:240-256)."""
    torch.manual_seed(0)
    e4m3 = torch.float8_e4m3fn
    if variant.startswith("a_m"):
        a = (torch.randn((K, M), device=device, dtype=torch.bfloat16) * 0.25).to(e4m3).transpose(0, 1)
    else:
        a = (torch.randn((M, K), device=device, dtype=torch.bfloat16) * 0.25).to(e4m3)
    if "_b_k" in variant:
        b = (torch.randn((N, K), device=device, dtype=torch.bfloat16) * 0.25).to(e4m3).transpose(0, 1)
    else:
        b = (torch.randn((K, N), device=device, dtype=torch.bfloat16) * 0.25).to(e4m3)
    return a, b


def run_variant(variant: str, warmup: int = 5) -> torch.Tensor:
    if variant not in VARIANTS:
        raise ValueError(f"variant must be one of {VARIANTS}, got {variant!r}")
    a, b = make_operands(variant)
    out = torch.empty((1, M, N), device="cuda", dtype=torch.bfloat16)
    scale = torch.tensor(0.5, device="cuda", dtype=torch.float32)

    def launch():
        bmm_scaled(a.unsqueeze(0), b.unsqueeze(0), out, scale_a=scale, sa_strides=(0, 0, 0), qbm=1,
                   scale_b=None, sb_strides=(0, 0, 0), qbn=1, qbk=K, bias=None, activation="none")

    for _ in range(warmup):
        launch()
    torch.cuda.synchronize()
    launch()
    torch.cuda.synchronize()
    reference = (a.float() @ b.float()) * scale
    torch.testing.assert_close(out[0].float(), reference.to(torch.bfloat16).float(), rtol=2e-2, atol=2e-2)
    return out[0]


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--variant", choices=VARIANTS, required=True)
    parser.add_argument("--warmup", type=int, default=5)
    args = parser.parse_args()
    run_variant(args.variant, args.warmup)
    print(f"fixed_{args.variant}_kernel completed: B=1 M={M} N={N} K={K} (libpcb200 scaled BMM, TMA operands)")


if __name__ == "__main__":
    main()
