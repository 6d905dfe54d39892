"""ctypes wrapper of the CPU checkers.  TEST INFRASTRUCTURE ONLY: imported by
tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs, never by the
product (tier_b200/).

  Oracle      -- oracle/libtkoracle.so, this repository's C restatement of the
                 reference arithmetic (tk_oracle.c, citations there).
  RefOracle   -- oracle/_ref/libtkref.so, the reference's own quant.h and
                 kernel bodies compiled from its sources (ref_harness.cpp);
                 absent when the reference tree was not available at build time.
  RefGPU      -- oracle/_ref/libtierref_gpu.so, the reference engine's GPU
                 linear path (fp3gemm / dq_k / gemv_q) compiled from tier.cpp
                 (ref_gpu.cu); timed beside libtierk by bench.py's reference arm.
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
P = ctypes.c_void_p


def _p(a: np.ndarray):
    return a.ctypes.data_as(P)


def reference_dir() -> Path | None:
    """The reference's tier/ directory: $TIER_REF, else the checkout beside
    this repository (../reference/tier); None when neither exists (the GPU box
    has no reference tree and uses the prebuilt _ref)."""
    import os
    env = os.environ.get("TIER_REF")
    cand = Path(env) if env else HERE.parent.parent / "reference" / "tier"
    return cand if (cand / "quant.h").exists() else None


def build(quiet: bool = True) -> None:
    """Run oracle/Makefile (compiles _ref too when the reference tree exists)."""
    ref = reference_dir()
    cmd = ["make", "-C", str(HERE)] + ([f"REF={ref}"] if ref else [])
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode:
        raise RuntimeError("oracle build failed:\n" + r.stdout + r.stderr)
    if not quiet:
        print(r.stdout)


class Oracle:
    def __init__(self):
        so = HERE / "libtkoracle.so"
        if not so.exists():
            build()
        L = ctypes.CDLL(str(so))
        L.tko_q_val.restype = ctypes.c_float
        L.tko_row_bytes.restype = ctypes.c_size_t
        L.tko_h2f.restype = ctypes.c_float
        L.tko_h2f.argtypes = [ctypes.c_uint16]
        L.tko_f2h.restype = ctypes.c_uint16
        L.tko_f2h.argtypes = [ctypes.c_float]
        L.tko_f2bf.restype = ctypes.c_uint16
        L.tko_f2bf.argtypes = [ctypes.c_float]
        self.L = L
        self.iq_grids = None
        try:
            self.set_iq_grids()
        except ImportError:
            pass            # no gguf-py: the IQ1/IQ2/IQ3 lattice types decode to NaN

    def set_iq_grids(self, grids: dict | None = None):
        """Register the lattice tables (int8, keyed as tier_b200.IQ_GRID_SHAPES);
        None takes them from gguf-py's IQ*.grid (the numbers of
        tier/quant_tables.h)."""
        from tier_b200 import IQ_GRID_SHAPES, iq_grids_from_gguf
        grids = iq_grids_from_gguf() if grids is None else grids
        self.iq_grids = [np.ascontiguousarray(grids[n], dtype=np.int8) for n, _, _ in IQ_GRID_SHAPES]
        self.L.tko_set_iq_grids(*[_p(a) for a in self.iq_grids])

    def row_bytes(self, qtype: int, cols: int) -> int:
        return int(self.L.tko_row_bytes(qtype, cols))

    def dequant(self, blocks: np.ndarray, qtype: int, rows: int, cols: int, out_dtype: int = 0,
                row_bytes: int | None = None) -> np.ndarray:
        rb = row_bytes or self.row_bytes(qtype, cols)
        b = np.ascontiguousarray(blocks, dtype=np.uint8)
        out = np.zeros((rows, cols), np.float32 if out_dtype == 0 else np.uint16)
        self.L.tko_dequant(_p(b), ctypes.c_size_t(rb), qtype, 0, rows, cols, out_dtype, _p(out))
        return out

    def gemv_warp_order(self, blocks, qtype, N, K, x):
        b = np.ascontiguousarray(blocks, dtype=np.uint8)
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.zeros(N, np.float32)
        self.L.tko_gemv_q_warp_order(_p(b), ctypes.c_size_t(self.row_bytes(qtype, K)), qtype, _p(x), _p(y), N, K)
        return y

    def qgemm_f64(self, blocks, qtype, N, K, X):
        b = np.ascontiguousarray(blocks, dtype=np.uint8)
        X = np.ascontiguousarray(X, dtype=np.float32)
        M = X.shape[0]
        Y = np.zeros((M, N), np.float64)
        self.L.tko_qgemm_f64(_p(b), ctypes.c_size_t(self.row_bytes(qtype, K)), qtype, _p(X), _p(Y), M, N, K)
        return Y

    def split3(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32)
        n = x.size
        h, m, l = (np.zeros(n, np.uint16) for _ in range(3))
        self.L.tko_split3_f16(_p(x), _p(h), _p(m), _p(l), ctypes.c_size_t(n))
        return h, m, l

    def dlogit(self, lg, rmax, rsum, labels, mask, v0, n_loss, cap):
        T, vc = lg.shape
        dl = np.zeros((T, vc), np.float32)
        self.L.tko_dlogit(_p(np.ascontiguousarray(lg, np.float32)), _p(np.ascontiguousarray(rmax, np.float64)),
                          _p(np.ascontiguousarray(rsum, np.float64)), _p(np.ascontiguousarray(labels, np.int32)),
                          _p(dl), T, vc, v0, n_loss, _p(np.ascontiguousarray(mask, np.uint8)), ctypes.c_float(cap))
        return dl

    def lse_chunk(self, lg, rmax, rsum, amax, tgt, labels, mask, v0):
        n_pred = rmax.size
        T, vc = lg.shape
        self.L.tko_lse_chunk(_p(np.ascontiguousarray(lg, np.float32)), _p(rmax), _p(rsum), _p(amax), _p(tgt),
                             _p(np.ascontiguousarray(labels, np.int32)), _p(np.ascontiguousarray(mask, np.uint8)),
                             n_pred, vc, v0)

    def lmhead_f64(self, W16: np.ndarray, X: np.ndarray, labels, mask, cap: float, chunk: int):
        """Whole two-pass LM head in fp64 (tier/tier.cpp:3184-3266).
        Returns (loss_sum, n_loss, amax[T-1], dX[T,H] float64)."""
        V, H = W16.shape
        T = X.shape[0]
        W16 = np.ascontiguousarray(W16, np.uint16)
        X = np.ascontiguousarray(X, np.float32)
        labels = np.ascontiguousarray(labels, np.int32)
        mask = np.ascontiguousarray(mask, np.uint8)
        loss = ctypes.c_double(0)
        n_loss = ctypes.c_int(0)
        amax = np.zeros(T - 1, np.int32)
        dX = np.zeros((T, H), np.float64)
        lg = np.zeros(T * min(chunk, V), np.float32)
        rmax = np.zeros(T - 1, np.float64)
        rsum = np.zeros(T - 1, np.float64)
        tgt = np.zeros(T - 1, np.float32)
        self.L.tko_lmhead_f64(_p(W16), V, H, _p(X), T, _p(labels), _p(mask), ctypes.c_float(cap), chunk,
                              ctypes.byref(loss), ctypes.byref(n_loss), _p(amax), _p(dX), _p(lg), _p(rmax),
                              _p(rsum), _p(tgt))
        return loss.value, n_loss.value, amax, dX, rmax, rsum, tgt


class RefOracle:
    """The reference's own code (quant.h, extracted kernel bodies) built in place."""

    SO = HERE / "_ref" / "libtkref.so"

    @classmethod
    def available(cls) -> bool:
        return cls.SO.exists()

    def __init__(self):
        L = ctypes.CDLL(str(self.SO))
        L.ref_q_val.restype = ctypes.c_float
        L.ref_row_bytes.restype = ctypes.c_size_t
        self.L = L

    def dequant(self, blocks, qtype, rows, cols, out_dtype=0):
        rb = int(self.L.ref_row_bytes(qtype, cols))
        b = np.ascontiguousarray(blocks, dtype=np.uint8)
        out = np.zeros((rows, cols), np.float32 if out_dtype == 0 else np.uint16)
        self.L.ref_dequant(_p(b), ctypes.c_size_t(rb), qtype, 0, rows, cols, out_dtype, _p(out))
        return out

    def quantize_row(self, qtype, x):
        x = np.ascontiguousarray(x, np.float32)
        rb = int(self.L.ref_row_bytes(qtype, x.size))
        o = np.zeros(rb, np.uint8)
        assert self.L.ref_q_row(qtype, _p(x), _p(o), x.size) == 1
        return o

    def split3(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32)
        n = x.size
        h, m, l = (np.zeros(n, np.uint16) for _ in range(3))
        self.L.ref_split3_fp16(_p(x), _p(h), _p(m), _p(l), ctypes.c_size_t(n))
        return h, m, l

    def lse_chunk(self, lg, rmax, rsum, amax, tgt, tokens, mask, v0):
        """lse_chunk_kernel itself (tier/tier.cpp:750-759) over rmax.size rows,
        blocks of 256 emulated threads; updates the state arrays in place."""
        n_pred = rmax.size
        T, vc = lg.shape
        self.L.ref_lse_chunk(_p(np.ascontiguousarray(lg, np.float32)), _p(rmax), _p(rsum), _p(amax), _p(tgt),
                             _p(np.ascontiguousarray(tokens, np.int32)), _p(np.ascontiguousarray(mask, np.uint8)),
                             n_pred, vc, v0)

    # -- the engine's own CPU GEMMs (tier/tier.cpp:1015-1099), extracted --
    def engine_pool(self, threads: int):
        """Start the reference's thread pool with `threads` workers."""
        self.L.ref_cpu_pool(int(threads))

    def dequant_bf16(self, blocks, qtype, n0, nrows, K, out=None):
        """q_val rows n0 .. n0+nrows rounded to bf16 (uint16 [nrows, K])."""
        b = np.ascontiguousarray(blocks, dtype=np.uint8)
        out = np.empty((nrows, K), np.uint16) if out is None else out
        rb = int(self.L.ref_row_bytes(qtype, K))
        self.L.ref_dequant_bf16(_p(b), ctypes.c_size_t(rb), qtype, n0, nrows, K, _p(out))
        return out

    def cpu_gemm_fwd(self, X, Wbf16, out=None):
        """cpu_gemm_fwd: out[M, N] = X[M, K] . W^T, W bf16 [N, K]."""
        M, K = X.shape
        N = Wbf16.shape[0]
        out = np.empty((M, N), np.float32) if out is None else out
        self.L.ref_cpu_gemm_fwd(_p(X), _p(Wbf16), _p(out), M, K, N)
        return out

    def cpu_gemm_dx(self, dY, Wbf16, out=None):
        """cpu_gemm_dx: out[M, K] = dY[M, N] . W, W bf16 [N, K]."""
        M, N = dY.shape
        K = Wbf16.shape[1]
        out = np.empty((M, K), np.float32) if out is None else out
        self.L.ref_cpu_gemm_dx(_p(dY), _p(Wbf16), _p(out), M, K, N)
        return out

    def qgemm_fwd(self, blocks, qtype, n0, nrows, K, X, threads):
        """CPU baseline: Y[M, nrows] via q_val row expansion + fp32 dots."""
        b = np.ascontiguousarray(blocks, dtype=np.uint8)
        X = np.ascontiguousarray(X, np.float32)
        M = X.shape[0]
        Y = np.zeros((M, nrows), np.float32)
        rb = int(self.L.ref_row_bytes(qtype, K))
        self.L.ref_cpu_qgemm_fwd(_p(b), ctypes.c_size_t(rb), qtype, n0, nrows, K, _p(X), M, _p(Y), nrows, threads)
        return Y

    def qgemm_dx(self, blocks, qtype, n0, nrows, K, dY, threads):
        b = np.ascontiguousarray(blocks, dtype=np.uint8)
        dY = np.ascontiguousarray(dY, np.float32)
        M = dY.shape[0]
        dX = np.zeros((M, K), np.float32)
        rb = int(self.L.ref_row_bytes(qtype, K))
        self.L.ref_cpu_qgemm_dx(_p(b), ctypes.c_size_t(rb), qtype, n0, nrows, K, _p(dY), dY.shape[1], M, _p(dX),
                                threads)
        return dX


class RefGPU:
    """The reference engine's own GPU functions (oracle/ref_gpu.cu) on device
    pointers (torch tensors' data_ptr()), on the legacy default stream."""

    SO = HERE / "_ref" / "libtierref_gpu.so"

    @classmethod
    def available(cls) -> bool:
        return cls.SO.exists()

    def __init__(self):
        L = ctypes.CDLL(str(self.SO))
        I, Z = ctypes.c_int, ctypes.c_size_t
        L.refgpu_fp3gemm_fwd.argtypes = [P, P, P, I, I, I]
        L.refgpu_fp3gemm_dx.argtypes = [P, P, P, I, I, I]
        L.refgpu_dequant_f16.argtypes = [P, I, Z, I, I, P]
        L.refgpu_gemv_q.argtypes = [P, I, Z, P, P, I, I]
        self.L = L

    @staticmethod
    def _ok(rc, what):
        if rc:
            raise RuntimeError(f"reference {what}: CUDA error {rc}")

    def fp3gemm_fwd(self, W16, X, Y, M, K, N):
        self._ok(self.L.refgpu_fp3gemm_fwd(W16.data_ptr(), X.data_ptr(), Y.data_ptr(), M, K, N), "fp3gemm fwd")

    def fp3gemm_dx(self, W16, dY, dX, M, K, N):
        self._ok(self.L.refgpu_fp3gemm_dx(W16.data_ptr(), dY.data_ptr(), dX.data_ptr(), M, K, N), "fp3gemm dx")

    def dequant_f16(self, W, qtype, rb, rows, cols, out):
        self._ok(self.L.refgpu_dequant_f16(W.data_ptr(), qtype, rb, rows, cols, out.data_ptr()), "dq_launch")

    def gemv_q(self, W, qtype, rb, x, y, N, K):
        self._ok(self.L.refgpu_gemv_q(W.data_ptr(), qtype, rb, x.data_ptr(), y.data_ptr(), N, K), "gemv_q")

    def sync(self):
        self._ok(self.L.refgpu_sync(), "sync")
