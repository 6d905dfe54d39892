"""The reference engine with its linear path on libtierk, run: one training
step of tierlm's own engine (tier/tier.cpp, built from its sources with the
integration/tier_bridge.h hooks) on a tiny random Llama, against the same
engine unhooked.  The losses must agree within 1e-3 (the step log prints four
decimals), and the hooked engine must have routed its layers' linear / dX
calls and both LM-head passes to libtierk (the bridge's own count).

The engines and the model come from `integration/e2e_tiny.py prepare`, run
where the reference tree is; without them the test is skipped."""
import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
BUILD = ROOT / "integration" / "_build"

pytestmark = pytest.mark.gpu


def test_hooked_engine_step_matches_reference_engine():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    need = [BUILD / "tier_ref", BUILD / "tier_tk", BUILD / "tiny" / "model.safetensors"]
    if not all(p.exists() for p in need):
        pytest.skip("engines not built (integration/e2e_tiny.py prepare)")
    r = subprocess.run([sys.executable, str(ROOT / "integration" / "e2e_tiny.py"), "run", "--tol", "1e-3"],
                       capture_output=True, text=True, timeout=900)
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert lines, r.stdout[-2000:] + r.stderr[-2000:]
    res = json.loads(lines[-1])
    assert res["abs_diff"] <= 1e-3, res
    for k in ("fwd", "dx", "lm_stats", "lm_grad"):
        assert res["routed_to_libtierk"].get(k, 0) > 0, res
    assert r.returncode == 0, res
