"""Engine integration, checked by building it: integration/build_patched_tier.py
adds the libtierk hooks (integration/tier_bridge.h) to the reference engine's
linear / linear_dx / linear_dx_acc (tier/tier.cpp:1202-1238) and chat_lin
(tier/tier.cpp:2351-2378), then compiles and links it with the reference's
own nvcc line.  The test needs the reference tree (skipped without it); the
binary is not run (it needs model files)."""
import os
import shutil
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT / "integration"))


def test_patch_hooks_each_call_site_once():
    from build_patched_tier import patch
    src = ("static void linear(hipblasHandle_t h, const float* x, const float* W, float* out, int M, int K, int N){ a; }\n"
           "static void linear_dx(hipblasHandle_t h, const float* dY, const float* W, float* dX, int M, int K, int N){ b; }\n"
           "static void linear_dx_acc(hipblasHandle_t h, const float* dY, const float* W, float* dX, int M, int K, int N)"
           "{ c; }\nstatic void chat_lin(ChatMat& m, const float* x, float* y, int M){ if(m.qt){ q; } else { r; } }\n"
           "int main(){ const int CHUNK=lm_chunk(seq_len);\n"
           "for(int v0=0; v0<VOCAB; v0+=CHUNK){ HIP_CHECK(hipMemcpy(d_chunk_bf,(const char*)head_h+(size_t)v0*row_bytes,"
           "(size_t)vc*row_bytes,hipMemcpyHostToDevice)); p1; }\n"
           "for(int v0=0; v0<VOCAB; v0+=CHUNK){ HIP_CHECK(hipMemcpy(d_chunk_bf,(const char*)head_h+(size_t)v0*row_bytes,"
           "(size_t)vc*row_bytes,hipMemcpyHostToDevice)); p2; } }\n")
    out = patch(src)
    assert out.count('#include "tier_bridge.h"') == 1
    assert "if(tk_bridge_fwd(x,W,out,M,K,N)) return; a;" in out
    assert "if(tk_bridge_dx(dY,W,dX,M,K,N,0.0f)) return; b;" in out
    assert "if(tk_bridge_dx(dY,W,dX,M,K,N,1.0f)) return; c;" in out
    assert "if(m.qt && tk_bridge_chat(m,W,x,y,M,g_chat_cs)){ } else if(m.qt){ q; }" in out
    assert "const int CHUNK=tk_bridge_lm_chunk(lm_chunk(seq_len));" in out
    i1, i2 = out.index("tk_bridge_lm_stats("), out.index("tk_bridge_lm_grad(")
    assert i1 < out.index("p1;") < i2 < out.index("p2;")
    with pytest.raises(SystemExit):
        patch(src.replace("linear_dx_acc", "other"))


def test_patched_engine_builds_and_binds_libtierk():
    from build_patched_tier import build, default_ref
    ref = default_ref()
    if not (ref / "tier.cpp").exists():
        pytest.skip("reference tree not present")
    if not (Path(os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")).exists() or shutil.which("nvcc")):
        pytest.skip("nvcc not available")
    from tier_b200 import build as tkbuild
    tkbuild.build()
    exe = build(ref)
    syms = subprocess.run(["nm", "-D", "--undefined-only", str(exe)], capture_output=True, text=True).stdout
    for name in ("tk_init", "tk_linear_fwd", "tk_linear_dx", "tk_gemv"):
        assert f" {name}\n" in syms, name
    deps = subprocess.run(["ldd", str(exe)], capture_output=True, text=True).stdout
    assert "libtierk.so" in deps


def test_bridge_routing_and_call_arguments(tmp_path):
    """integration/tier_bridge.h with stand-ins for the engine's globals and
    recording stubs for the library (tests/bridge_check.cpp): which weights go
    to libtierk, the argument order of each call (leading dimensions, beta,
    product set, stream, TK_WFROZEN only for resident weights), and the
    fall-back to the reference path when a call fails."""
    if not shutil.which("g++"):
        pytest.skip("g++ not available")
    exe = tmp_path / "bridge_check"
    r = subprocess.run(["g++", "-std=c++17", "-Wall", "-Wextra", "-Werror", "-I", str(ROOT / "include"),
                        "-I", str(ROOT / "integration"), str(ROOT / "tests" / "bridge_check.cpp"), "-o", str(exe)],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stderr
    lines = [ln.split() for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 17
    assert all(v == "1" for _, v in lines), [n for n, v in lines if v != "1"]


def test_tiny_model_is_accepted_by_the_reference_arch_tool(tmp_path):
    """integration/e2e_tiny.py's model: a random 2-layer Llama that the
    reference's own arch.py describes (tier_arch.txt), plus the token file the
    engine's training mode reads (seq_len int32 ids)."""
    from build_patched_tier import default_ref
    ref = default_ref()
    if not (ref / "arch.py").exists():
        pytest.skip("reference tree not present")
    pytest.importorskip("transformers")
    from e2e_tiny import SEQ, make_model
    make_model(tmp_path, ref)
    desc = (tmp_path / "tier_arch.txt").read_text()
    for key in ("family llama", "hidden 256", "inter 512", "heads 4", "vocab 2048", "head lm_head.weight"):
        assert key in desc, key
    assert (tmp_path / "tokens.bin").stat().st_size == 4 * SEQ
