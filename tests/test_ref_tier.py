"""The CUDA tier inside the reference's own kernel table.

oracle/tlm_kern_cuda.c is the reference-side binding a maintainer of the
reference would add next to tlm_kern_avx512.c (its fill function fills the
tlm_quant_kernels table, src/lib/tlm_quant.h:146-171, with libtlmg's host
adapters). oracle/ref_tier.c runs on that table, unchanged, the reference's
start-up self-test (selftest_tier, src/lib/tlm_quant.c:1014-1056) and the
tier matrix of its unit tests (test_tiers_bitexact / test_matvec_tiles,
tests/test_quant.c:708-864): every result must be the scalar tier's bits.
"""
from __future__ import annotations

import re
import subprocess
from pathlib import Path

import pytest

CHECK = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "bin" / "cuda_tier_check"


@pytest.mark.gpu
@pytest.mark.skipif(not CHECK.exists(), reason="oracle/_ref not built (make -C oracle gate)")
def test_reference_selftest_and_tier_matrix_on_cuda_tier():
    r = subprocess.run([str(CHECK)], capture_output=True, text=True, timeout=600)
    out = r.stdout + r.stderr
    assert r.returncode == 0, out[-4000:]
    m = re.search(r"selftest_tier cuda: (\d+) entries filled, (\d+) failed", out)
    assert m and int(m.group(1)) == 9 and int(m.group(2)) == 0, out
    m = re.search(r"bit-exact single-row comparisons: (\d+), mismatches: (\d+)", out)
    assert m and int(m.group(1)) > 3000 and int(m.group(2)) == 0, out
    m = re.search(r"bit-exact matvec rows vs scalar: (\d+), mismatches: (\d+)", out)
    assert m and int(m.group(1)) > 1000 and int(m.group(2)) == 0, out
    assert "tier matrix cuda: 0 failure(s)" in out, out
