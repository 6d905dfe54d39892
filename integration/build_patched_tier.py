#!/usr/bin/env python3
"""Build tierlm's engine (tier/tier.cpp) with its frozen-weight linear path
routed through libtierk.so -- the integration a maintainer would make, checked
by compiling and linking it.

The recipe reads tier/tier.cpp where it lies and adds four hooks:
  * `#include "tier_bridge.h"` just before `linear` (tier/tier.cpp:1202);
  * a first statement in `linear`, `linear_dx` and `linear_dx_acc`
    (tier/tier.cpp:1202-1238) that hands fp16-x3 weights to tk_linear_fwd /
    tk_linear_dx and returns;
  * in `chat_lin` (tier/tier.cpp:2351), the quantized branch tries tk_gemv /
    tk_linear_fwd first;
  * in the LM head (tier/tier.cpp:3184-3266), the chunk size is rounded to 256
    rows and each chunk of the two vocabulary loops tries tk_lmhead_stats /
    tk_lmhead_grad right after its rows reach the device.
It writes the patched engine to integration/_build/tier_tk.cpp (build output:
git-ignored, never committed) and compiles it
with the reference's own nvcc line (tier/build.sh:89) for sm_100, linked to
libtierk.so.  The binary is not run here: it needs model files.

usage: python integration/build_patched_tier.py [REF_DIR]
       (REF_DIR defaults to $TIER_REF, else the reference checkout beside this
        repository, ../reference/tier)
"""
from __future__ import annotations

import os
import re
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
OUT_DIR = ROOT / "integration" / "_build"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")


def default_ref() -> Path:
    env = os.environ.get("TIER_REF")
    return Path(env) if env else ROOT.parent / "reference" / "tier"


# (pattern, replacement builder, what it hooks).  Each pattern must match once.
def _after(stmt):
    return lambda m: m.group(0) + stmt


HOOKS = [
    (r"static void linear\(hipblasHandle_t h, const float\* x, const float\* W, float\* out, int M, int K, int N\)\{",
     lambda m: '#include "tier_bridge.h"\n' + m.group(0) + " if(tk_bridge_fwd(x,W,out,M,K,N)) return;",
     "linear"),
    (r"static void linear_dx\(hipblasHandle_t h, const float\* dY, const float\* W, float\* dX, int M, int K, int N\)\{",
     _after(" if(tk_bridge_dx(dY,W,dX,M,K,N,0.0f)) return;"), "linear_dx"),
    (r"static void linear_dx_acc\(hipblasHandle_t h, const float\* dY, const float\* W, float\* dX, int M, int K, "
     r"int N\)\{", _after(" if(tk_bridge_dx(dY,W,dX,M,K,N,1.0f)) return;"), "linear_dx_acc"),
]
# chat_lin: the first `if(m.qt){` after its signature becomes
# `if(m.qt && tk_bridge_chat(...)){ } else if(m.qt){`
CHAT_SIG = r"static void chat_lin\(ChatMat& m, const float\* x, float\* y, int M\)\{"
CHAT_QT = r"if\(m\.qt\)\{"


# The LM head: the chunk size, and the statement that uploads a chunk, which
# opens both vocabulary loops (pass 1, then pass 2).
LM_CHUNK = "const int CHUNK=lm_chunk(seq_len);"
LM_UPLOAD = ("HIP_CHECK(hipMemcpy(d_chunk_bf,(const char*)head_h+(size_t)v0*row_bytes,(size_t)vc*row_bytes,"
             "hipMemcpyHostToDevice));")
LM_PASS1 = (" if(!g_gen && g_fp16_storage && n_pred>0 && tk_bridge_lm_stats(d_chunk_bf,v0,vc,HIDDEN,normed_final,"
            "seq_len,d_tokens,d_lmask,SOFTCAP,d_running_max,d_running_sum,d_amax,d_tgt)){ if(g_prog && !g_is_ev) "
            "printf(\"prog h %d\\n\", v0/CHUNK+1); continue; }")
LM_PASS2 = (" if(g_fp16_storage && tk_bridge_lm_grad(d_chunk_bf,v0,vc,HIDDEN,normed_final,seq_len,d_tokens,d_lmask,"
            "n_loss,SOFTCAP,d_running_max,d_running_sum,d_normed_final)){ if(g_prog && !g_is_ev) "
            "printf(\"prog g %d\\n\", v0/CHUNK+1); continue; }")


def patch_lm_head(src: str) -> str:
    if src.count(LM_CHUNK) != 1:
        raise SystemExit(f"hook 'lm_chunk': expected one match, found {src.count(LM_CHUNK)}")
    src = src.replace(LM_CHUNK, "const int CHUNK=tk_bridge_lm_chunk(lm_chunk(seq_len));")
    if src.count(LM_UPLOAD) != 2:
        raise SystemExit(f"hook 'lm head loops': expected two chunk uploads, found {src.count(LM_UPLOAD)}")
    i = src.index(LM_UPLOAD) + len(LM_UPLOAD)
    src = src[:i] + LM_PASS1 + src[i:]
    j = src.index(LM_UPLOAD, i) + len(LM_UPLOAD)
    return src[:j] + LM_PASS2 + src[j:]


def patch(src: str) -> str:
    for pat, rep, name in HOOKS:
        hits = re.findall(pat, src)
        if len(hits) != 1:
            raise SystemExit(f"hook '{name}': expected one match, found {len(hits)}")
        src = re.sub(pat, rep, src, count=1)
    m = re.search(CHAT_SIG, src)
    if not m:
        raise SystemExit("hook 'chat_lin': signature not found")
    q = re.compile(CHAT_QT).search(src, m.end())
    if not q:
        raise SystemExit("hook 'chat_lin': quantized branch not found")
    src = src[:q.start()] + "if(m.qt && tk_bridge_chat(m,W,x,y,M,g_chat_cs)){ } else if(m.qt){" + src[q.end():]
    return patch_lm_head(src)


def build(ref: Path, hooked: bool = True) -> Path:
    """Build the engine into integration/_build/: tier_tk (hooked, linked to
    libtierk.so) or, with hooked=False, tier_ref (the reference unchanged,
    compiled from tier.cpp where it lies with the same command line)."""
    tier = ref / "tier.cpp"
    if not tier.exists():
        raise SystemExit(f"{tier} not found")
    lib = ROOT / "tier_b200" / "libtierk.so"
    if hooked and not lib.exists():
        raise SystemExit("libtierk.so not built: python -m tier_b200.build")
    OUT_DIR.mkdir(parents=True, exist_ok=True)
    if hooked:
        src = OUT_DIR / "tier_tk.cpp"
        src.write_text(patch(tier.read_text()))
        exe = OUT_DIR / "tier_tk"
    else:
        src, exe = tier, OUT_DIR / "tier_ref"
    cmd = [NVCC, "-x", "cu", "-DTIER_CUDA", "-std=c++17", "-O1", "-Xcompiler", "-pthread -Wno-unused-result",
           "-diag-suppress", "177,1650", "-I", str(ref), "-I", str(ROOT / "include"), "-I", str(ROOT / "integration"),
           "-gencode", "arch=compute_100,code=sm_100", str(src), "-o", str(exe), "-lcublas", "-lcublasLt"]
    if hooked:
        cmd += ["-L", str(lib.parent), "-ltierk", "-Xlinker", f"-rpath={lib.parent}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode:
        sys.stderr.write(r.stdout[-4000:] + r.stderr[-4000:])
        raise SystemExit("engine did not build")
    return exe


if __name__ == "__main__":
    print(build(Path(sys.argv[1]) if len(sys.argv) > 1 else default_ref()))
