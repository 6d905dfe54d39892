"""The decode of the table-level block types (IQ4_NL, IQ4_XS, MXFP4, NF4, FP4,
TQ1_0, TQ2_0; tier_b200/csrc/tk_qtypes.h) and of the lattice types (IQ2_XXS,
IQ2_XS, IQ2_S, IQ3_XXS, IQ3_S, IQ1_S, IQ1_M; tk_qgrid.h) -- the headers the GPU
kernels include -- compiled for the host and checked bit-for-bit: against the
golden vectors (gguf-py 0.19.0 and the reference's quant.h, tier/quant.h:69-73,
91-119), against the reference's q_val itself on fresh random blocks when
oracle/_ref is built, and against the CPU oracle's restatement.  The lattice
tables come from gguf-py (the numbers of tier/quant_tables.h)."""
import ctypes
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

from conftest import GOLDEN

ROOT = Path(__file__).resolve().parent.parent
DQ = np.load(GOLDEN / "dequant_golden.npz")
TABLE_TYPES = {"IQ4_NL": 20, "IQ4_XS": 23, "TQ1_0": 34, "TQ2_0": 35, "MXFP4": 39, "NF4": 200, "FP4": 201}
GEOM = {20: (32, 18), 23: (256, 136), 34: (256, 54), 35: (256, 66), 39: (32, 17), 200: (64, 36), 201: (64, 36)}
GRID_TYPES = {"IQ2_XXS": 16, "IQ2_XS": 17, "IQ2_S": 22, "IQ3_XXS": 18, "IQ3_S": 21, "IQ1_S": 19, "IQ1_M": 29}
GRID_GEOM = {16: 66, 17: 74, 22: 82, 18: 98, 21: 110, 19: 50, 29: 56}


@pytest.fixture(scope="module")
def host(tmp_path_factory):
    cxx = shutil.which("g++")
    if not cxx:
        pytest.skip("g++ not available")
    so = tmp_path_factory.mktemp("qtypes") / "libqtypes_host.so"
    r = subprocess.run([cxx, "-O2", "-std=c++17", "-shared", "-fPIC", "-I", str(ROOT / "tier_b200" / "csrc"),
                        str(ROOT / "tests" / "qtypes_host.cpp"), "-o", str(so)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    lib = ctypes.CDLL(str(so))
    lib.tkq_host_half.restype = ctypes.c_float
    return lib


@pytest.fixture(scope="module")
def tab(host):
    """The library's table buffer layout, filled from gguf-py."""
    pytest.importorskip("gguf")
    from tier_b200 import IQ_GRID_SHAPES, iq_grids_from_gguf
    g = iq_grids_from_gguf()
    buf = np.zeros(host.tkq_host_grid_offset(7), np.int8)
    for w, (name, rows, cols) in enumerate(IQ_GRID_SHAPES):
        o = host.tkq_host_grid_offset(w)
        buf[o:o + rows * cols] = g[name].reshape(-1)
    host.tkq_host_fill_signs(buf.ctypes.data_as(ctypes.c_void_p))
    return buf


def dequant_grid(lib, tab, b, t, rows, cols):
    out = np.zeros((rows, cols), np.float32)
    b = np.ascontiguousarray(b)
    lib.tkq_host_dequant_grid(b.ctypes.data_as(ctypes.c_void_p), ctypes.c_size_t(b.shape[1]), t, rows, cols,
                              tab.ctypes.data_as(ctypes.c_void_p), out.ctypes.data_as(ctypes.c_void_p))
    return out


def grid_blocks(rng, t, rows, cols):
    nb = rows * cols // 256
    b = rng.integers(0, 256, size=(nb, GRID_GEOM[t]), dtype=np.uint8)
    h = (rng.standard_normal(nb) * 0.02).astype(np.float16).view(np.uint16)
    if t == 29:      # IQ1_M: fp16 scale in the top nibbles of the four scale words
        sc = b[:, 48:56].copy().view(np.uint16).reshape(nb, 4)
        for k in range(4):
            sc[:, k] = (sc[:, k] & 0x0FFF) | (((h >> (4 * k)) & 0xF) << 12)
        b[:, 48:56] = sc.view(np.uint8).reshape(nb, 8)
    else:
        b[:, 0:2] = h.view(np.uint8).reshape(nb, 2)
    return b.reshape(rows, -1).copy()


def dequant(lib, b, t, rows, cols):
    out = np.zeros((rows, cols), np.float32)
    b = np.ascontiguousarray(b)
    lib.tkq_host_dequant(b.ctypes.data_as(ctypes.c_void_p), ctypes.c_size_t(b.shape[1]), t, rows, cols,
                         out.ctypes.data_as(ctypes.c_void_p))
    return out


def random_blocks(rng, t, rows, cols):
    be, bb = GEOM[t]
    nb = rows * cols // be
    b = rng.integers(0, 256, size=(nb, bb), dtype=np.uint8)
    if t in (200, 201):
        b[:, 0:4] = np.abs(rng.standard_normal(nb) * 0.05).astype(np.float32).view(np.uint8).reshape(nb, 4)
    elif t != 39:
        off = {20: 0, 23: 0, 34: 52, 35: 64}[t]
        b[:, off:off + 2] = (rng.standard_normal(nb) * 0.02).astype(np.float16).view(np.uint8).reshape(nb, 2)
    return b.reshape(rows, -1).copy()


def test_geometry(host):
    e, b = ctypes.c_int(), ctypes.c_int()
    for t, (ee, bb) in GEOM.items():
        assert host.tkq_host_geom(t, ctypes.byref(e), ctypes.byref(b)) == 1
        assert (e.value, b.value) == (ee, bb)
    assert host.tkq_host_geom(16, ctypes.byref(e), ctypes.byref(b)) == 0      # IQ2_XXS: not a table type


def test_half_conversion_exhaustive(host):
    h = np.arange(65536, dtype=np.uint32)
    got = np.array([host.tkq_host_half(int(v)) for v in h], np.float32)
    want = h.astype(np.uint16).view(np.float16).astype(np.float32)
    nan = np.isnan(want)
    assert np.array_equal(got[~nan].view(np.uint32), want[~nan].view(np.uint32))
    assert np.isnan(got[nan]).all()


@pytest.mark.parametrize("name", sorted(TABLE_TYPES))
def test_golden_bit_exact(host, name):
    b, want = DQ[f"{name}_blocks"], DQ[f"{name}_f32"]
    got = dequant(host, b, TABLE_TYPES[name], *want.shape)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), name


@pytest.mark.parametrize("t", sorted(GEOM))
def test_reference_q_val_random(host, t):
    from oracle.oracle import RefOracle
    if not RefOracle.available():
        pytest.skip("oracle/_ref not built (reference tree absent)")
    rng = np.random.default_rng(100 + t)
    b = random_blocks(rng, t, 16, 1024)
    got = dequant(host, b, t, 16, 1024)
    want = RefOracle().dequant(b, t, 16, 1024)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("t", sorted(GEOM))
def test_oracle_port_agrees(host, oracle, t):
    rng = np.random.default_rng(200 + t)
    b = random_blocks(rng, t, 8, 512)
    assert np.array_equal(dequant(host, b, t, 8, 512).view(np.uint32), oracle.dequant(b, t, 8, 512).view(np.uint32))


def test_sign_table_rule(host, tab):
    from gguf import quants
    off = host.tkq_host_grid_offset(6)
    assert np.array_equal(tab[off:off + 128].view(np.uint8), np.frombuffer(quants.IQ2_XXS.ksigns, np.uint8))


@pytest.mark.parametrize("name", sorted(GRID_TYPES))
def test_grid_golden_bit_exact(host, tab, name):
    b, want = DQ[f"{name}_blocks"], DQ[f"{name}_f32"]
    got = dequant_grid(host, tab, b, GRID_TYPES[name], *want.shape)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), name


@pytest.mark.parametrize("t", sorted(GRID_GEOM))
def test_grid_reference_q_val_random(host, tab, t):
    from oracle.oracle import RefOracle
    if not RefOracle.available():
        pytest.skip("oracle/_ref not built (reference tree absent)")
    rng = np.random.default_rng(700 + t)
    b = grid_blocks(rng, t, 16, 1024)
    want = RefOracle().dequant(b, t, 16, 1024)
    assert np.array_equal(dequant_grid(host, tab, b, t, 16, 1024).view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("t", sorted(GRID_GEOM))
def test_grid_oracle_port_agrees(host, tab, oracle, t):
    rng = np.random.default_rng(800 + t)
    b = grid_blocks(rng, t, 8, 512)
    got = dequant_grid(host, tab, b, t, 8, 512)
    assert np.array_equal(got.view(np.uint32), oracle.dequant(b, t, 8, 512).view(np.uint32))
