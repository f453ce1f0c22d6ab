"""The exact scalar helpers of the kernels (RMSNorm reciprocal root, probability division), compiled
for the host from the same header and checked against exact integer references (CPU only)."""
import os
import shutil
import subprocess

import pytest

from conftest import PKG, REPO


@pytest.mark.skipif(shutil.which("nvcc") is None, reason="nvcc not available")
def test_exact_helpers_match_integer_references(tmp_path):
    exe = str(tmp_path / "exact_helpers_check")
    src = os.path.join(REPO, "tests", "exact_helpers_check.cu")
    # device code in the included headers is built for the engine's target; only host code runs here
    subprocess.check_call(["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O2", "-std=c++17",
                           "-I" + os.path.join(PKG, "csrc"), "-o", exe, src])
    r = subprocess.run([exe, "300000"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "mismatches 0" in r.stdout
