"""The reference's fixed-shape ``--variant`` microbench on libpcb200: every
variant runs and passes the reference's own check (rtol = atol = 2e-2 against
``(A.float() @ B.float()) * scale`` in bf16, profile_fixed_b_n.py:277-283)."""

import subprocess
import sys

import pytest

from practice_cuda_b200.microbench import VARIANTS, run_variant

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("variant", VARIANTS)
def test_variant(variant):
    out = run_variant(variant, warmup=2)
    assert out.shape == (64, 64)


def test_cli():
    r = subprocess.run([sys.executable, "-m", "practice_cuda_b200.microbench", "--variant", "a_m_b_n"],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "fixed_a_m_b_n_kernel completed" in r.stdout
