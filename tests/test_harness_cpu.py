"""The reference's own plugin registry sees this library's implementations.

``practice_cuda_b200.registry.install_into`` registers every ``b200_*`` quant
and BMM impl into the reference's ``fp8_bench.registry``
(``fp8_training/fp8_bench/registry.py:116-209``), which its harnesses
(``bench_quant``, ``bench_bmm``, ``profile_one``) enumerate.  Needs the
reference's Python package: the install under ``baseline/_ref`` (a copy of
its ``fp8_bench`` tree) or a checkout; skipped when neither is present.
No GPU: nothing is launched."""

import os
import subprocess
import sys
import textwrap

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CANDIDATES = [os.path.join(ROOT, "baseline", "_ref"), "/root/reference/fp8_training"]


def _ref_path():
    for p in CANDIDATES:
        if os.path.isdir(os.path.join(p, "fp8_bench")):
            return p
    return None


@pytest.mark.skipif(_ref_path() is None, reason="the reference's fp8_bench package is not installed here")
def test_install_into_reference_registry():
    # A fresh interpreter keeps the reference's modules out of this test process.
    code = textwrap.dedent(f"""
        import sys
        sys.path[:0] = [{ROOT!r}, {_ref_path()!r}]
        import fp8_bench.registry as ref
        from practice_cuda_b200 import registry as ours
        installed = ours.install_into(ref)
        names = ref.bmm_impl_names()
        assert "b200_per_block_1x128_128x128_a_k_b_n" in installed
        assert "triton_per_block_1d_a_k_b_n" in names  # the reference's own impls stay
        for n in installed:
            if n in ref.BMM_IMPLS:
                a, b = ref.BMM_IMPLS[n], ours.BMM_IMPLS[n]
                assert n in names
                assert type(a) is ref.BMMImpl
                assert (a.quant_impl, a.layout, a.a_layout, a.quant_a_kwargs, a.quant_b_kwargs) == \\
                       (b.quant_impl, b.layout, b.a_layout, b.quant_a_kwargs, b.quant_b_kwargs)
                assert a.quant_impl in ref.QUANT_IMPLS
            else:
                assert type(ref.QUANT_IMPLS[n]) is ref.QuantImpl
        # installing twice is a no-op
        assert ours.install_into(ref) == []
        print(len(installed))
    """)
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-3000:]
    assert int(r.stdout.strip().splitlines()[-1]) > 30
