"""The branch-free exact Q8 quantisation (gemv_device.cuh: q8_scale,
q8_code_r) against CUDA's own IEEE division and roundf, the reference's
arithmetic (matmul.cu:18-19): every non-negative float as a group maximum
for the scale, and every mantissa of the maximum at exponents across the
float range with values at, beside and between the code boundaries. The
checker is tests/cuda/q8_exact_test.cu, compiled here with nvcc."""
import os
import subprocess

import pytest

from conftest import PKG, ROOT

pytestmark = pytest.mark.gpu


def test_q8_helpers_match_ieee_bit_for_bit(cuda, tmp_path):
    src = os.path.join(ROOT, "tests", "cuda", "q8_exact_test.cu")
    exe = str(tmp_path / "q8_exact_test")
    subprocess.run(["nvcc", "-std=c++17", "-O3", "-gencode", "arch=compute_100a,code=sm_100a",
                    "-I" + os.path.join(PKG, "csrc"), "-I" + os.path.join(ROOT, "include"), src, "-o", exe],
                   check=True, capture_output=True, text=True)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=600)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "0 mismatches; codes" in r.stdout and r.stdout.strip().endswith("0 mismatches")
