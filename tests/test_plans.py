"""The decode GEMV launch plans, checked on the host: tests/plan_check.cu
includes the kernel sources, sweeps block types, K, N and token counts, and
asserts the shared-memory, alignment and bank-stride invariants of every plan
(a plan that broke them would fault on the GPU)."""
import os
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def test_decode_gemv_plans(tmp_path):
    nvcc = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
    if not (Path(nvcc).exists() or shutil.which("nvcc")):
        pytest.skip("nvcc not available")
    exe = tmp_path / "plan_check"
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O1", "-std=c++17", "--expt-relaxed-constexpr",
           "-I", str(ROOT / "include"), "-I", str(ROOT / "tier_b200" / "csrc"),
           str(ROOT / "tests" / "plan_check.cu"), "-o", str(exe)]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "0 failures" in r.stdout
