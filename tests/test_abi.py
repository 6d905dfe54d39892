"""The C ABI library builds, loads, and exports exactly what include/tierk.h
declares; host-side validation works without a GPU."""
import ctypes
import re
import subprocess

import pytest

from conftest import ROOT


def declared_symbols():
    text = (ROOT / "include" / "tierk.h").read_text()
    return sorted(set(re.findall(r"\b(tk_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from tier_b200 import build
    build.build()
    import tier_b200
    return tier_b200.load()


def test_every_declared_symbol_is_exported(lib):
    so = ROOT / "tier_b200" / "libtierk.so"
    out = subprocess.run(["nm", "-D", "--defined-only", str(so)], capture_output=True, text=True).stdout
    exported = {l.split()[-1] for l in out.splitlines() if " T " in l}
    missing = [s for s in declared_symbols() if s not in exported]
    assert not missing, missing
    assert all(s.startswith("tk_") for s in exported), "only the tk_* C ABI may be exported"


def test_binding_covers_header():
    import tier_b200
    bound = {name for name, _, _ in tier_b200.SIGNATURES}
    assert bound == set(declared_symbols())


def test_row_bytes_matches_oracle(lib, oracle):
    import tier_b200 as tk
    assert len(tk.QTYPES) == 27                     # every type of tier/quant.h:25-31
    for t in sorted(tk.QTYPES.values()):
        for cols in (256, 4096, 5120, 14336):
            assert lib.tk_row_bytes(t, cols) == oracle.row_bytes(t, cols), (t, cols)
    assert lib.tk_row_bytes(12, 100) == 0          # not a block multiple
    assert lib.tk_row_bytes(99, 256) == 0          # unknown type


def test_null_context_is_rejected_not_crashed(lib):
    st = lib.tk_dequant(None, 8, None, 0, 0, 1, 32, 0, None, None)
    assert st == 1  # TK_ERR_INVALID
    assert b"null context" in lib.tk_last_error_string()
    st = lib.tk_gemv(None, 8, None, 34, 1, 32, None, 32, 1, None, 1, None)
    assert st == 1
    st = lib.tk_gemv_multi(None, 8, 2, None, None, None, None, 34, 32, None, 32, 1, None)
    assert st == 1 and b"null context" in lib.tk_last_error_string()
    st = lib.tk_set_iq_grids(None, None)
    assert st == 1 and b"null context" in lib.tk_last_error_string()
    # the peer collectives refuse a null context and an unconnected one alike
    assert lib.tk_allgather(None, None, 16, None, None) == 1
    assert lib.tk_allreduce_f32(None, None, 4, None) == 1
    assert lib.tk_lmhead_merge(None, 4, None, None, None, None, None, 0, None) == 1
    # forward + dX in one launch, plain and reduce-scattered
    for fn in (lib.tk_linear_fwd_dx, lib.tk_linear_fwd_dx_rs):
        assert fn(None, None, None, 0, 256, 64, None, 64, None, 0, 256, 64, None, 64, 0, None) == 1
        assert b"null context" in lib.tk_last_error_string()


def test_qtype_values_and_names_match_header(lib):
    """Every TK_<type> enum of the header equals the Python constant, and the
    library's name table maps the same names to the same codes."""
    import tier_b200 as tk
    text = (ROOT / "include" / "tierk.h").read_text()
    for name, code in tk.QTYPES.items():
        m = re.search(rf"\bTK_{name}\s*=\s*(\d+)", text)
        assert m and int(m.group(1)) == code, name
        assert lib.tk_qtype_from_name(name.encode()) == code, name
        assert lib.tk_qtype_name(code) == name.encode(), name


def test_flag_values_match_header():
    """The Python flag constants equal the header's enums."""
    import tier_b200 as tk
    text = (ROOT / "include" / "tierk.h").read_text()
    for name, value in (("TK_QFUSED", tk.QFUSED), ("TK_WFROZEN", tk.WFROZEN), ("TK_WREUSE", tk.WREUSE),
                        ("TK_IPC_HANDLE_BYTES", tk.IPC_HANDLE_BYTES)):
        m = re.search(rf"\b{name}\s*=\s*(0x[0-9a-fA-F]+|\d+)", text)
        assert m and int(m.group(1), 0) == value, name
    flags = [tk.QFUSED, tk.WREUSE]                  # OR-ed into `products` with the product set (0..4)
    assert all(f & 0xff == 0 for f in flags) and tk.QFUSED & tk.WREUSE == 0


def test_init_without_gpu_reports_error(lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    h = ctypes.c_void_p()
    st = lib.tk_init(0, ctypes.byref(h))
    assert st != 0 and not h.value
    assert lib.tk_last_error_string()


def test_product_sets_and_types_exposed():
    import tier_b200 as tk
    assert (tk.X3_AUTO, tk.X3_REF, tk.X3_HHL, tk.X2, tk.X1) == (0, 1, 2, 3, 4)
    assert tk.Q8_0 == 8 and tk.Q4_K == 12 and tk.Q5_K == 13   # tier/quant.h:20-23


def test_plain_c_caller(lib, tmp_path):
    """include/tierk.h compiles as strict C99 and a C program linked to
    libtierk.so gets the same answers as the Python binding (no GPU needed)."""
    import shutil
    import tier_b200 as tk
    if not shutil.which("gcc"):
        pytest.skip("gcc not available")
    exe = tmp_path / "abi_consumer"
    so_dir = ROOT / "tier_b200"
    r = subprocess.run(["gcc", "-std=c99", "-pedantic", "-Wall", "-Wextra", "-Werror", "-I", str(ROOT / "include"),
                        str(ROOT / "tests" / "abi_consumer.c"), "-L", str(so_dir), "-ltierk",
                        f"-Wl,-rpath,{so_dir}", "-o", str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    lines = r.stdout.split("\n")
    rows = [ln.split() for ln in lines if ln.startswith("type ")]
    assert len(rows) == 27
    for _, code, name, rb, back in rows:
        assert tk.QTYPES[name] == int(code) == int(back)
        assert int(rb) == tk.row_bytes(int(code), 4096)
    assert "null_ctx 1 1" in lines and "null_grids 1" in lines
    init = next(ln for ln in lines if ln.startswith("init "))
    import torch
    if not torch.cuda.is_available():
        assert init != "init 0 1" and init.endswith(" 1")     # an error status, no context


def test_lmhead_chunk_follows_the_reference_rule(lib):
    """tk_lmhead_chunk = tier/tier.cpp:2015-2017 (total memory / 36 / (6H + 8T),
    clamped to [1024, V]) rounded down to 256 rows instead of 128."""
    import tier_b200 as tk

    def ref_rule(total, H, T, V):             # the reference's arithmetic, then our 256 rounding
        if total == 0:
            return 8192
        c = total // 36 // (H * 6 + max(T, 1) * 8)
        c = c // 128 * 128
        return max(1024, min(c // 256 * 256, (V + 255) // 256 * 256))

    b200 = 183359 * 2 ** 20
    assert tk.lmhead_chunk(b200, 3840, 8192, 262144) == 60160        # C4's shape on a B200's 183,359 MiB
    for total in (0, 2 ** 30, 24 * 2 ** 30, 80 * 2 ** 30, b200):
        for H, T, V in ((3840, 8192, 262144), (5120, 4096, 152064), (2048, 1, 32000), (4096, 65536, 1000)):
            got = tk.lmhead_chunk(total, H, T, V)
            assert got == ref_rule(total, H, T, V), (total, H, T, V)
            assert got % 256 == 0 or total == 0
