"""Build libtierk.so in-tree: every .cu under tier_b200/csrc compiled for
sm_100a only (tcgen05/TMA need the arch-specific target) and linked into one
shared library beside this file.

usage: python -m tier_b200.build [--force] [-v]
"""
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
OUT = PKG / "libtierk.so"
BUILD = PKG.parent / "_build"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
         "--expt-relaxed-constexpr", "-I", str(PKG.parent / "include")]


def sources():
    return sorted(CSRC.glob("*.cu"))


def deps():
    return sources() + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [PKG.parent / "include" / "tierk.h"]


def up_to_date() -> bool:
    if not OUT.exists():
        return False
    t = OUT.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in deps())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return OUT
    BUILD.mkdir(exist_ok=True)
    objs = []
    procs = []
    for src in sources():
        obj = BUILD / (src.stem + ".o")
        cmd = [NVCC, *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
            print(" ".join(cmd))
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
        objs.append(obj)
    failed = False
    for src, p in procs:
        out, _ = p.communicate()
        if out.strip():
            sys.stderr.write(out)
        if p.returncode:
            sys.stderr.write(f"nvcc failed on {src.name}\n")
            failed = True
    if failed:
        raise RuntimeError("libtierk build failed")
    # export only the C ABI (tk_*); every other symbol stays local
    vscript = BUILD / "tierk.map"
    vscript.write_text("{ global: tk_*; local: *; };\n")
    tmp = OUT.with_suffix(".so.tmp")
    link = [NVCC, *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-Xlinker", f"--version-script={vscript}",
            "-lcudart_static", "-ldl", "-lpthread", "-lrt"]
    r = subprocess.run(link, capture_output=True, text=True)
    if r.returncode:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("libtierk link failed")
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(OUT)
