"""tier_b200 -- B200-native (sm_100a) frozen-weight linear path of tierlm.

The product is the C ABI in include/tierk.h, implemented by libtierk.so (built
in-tree by ``python -m tier_b200.build``).  This module is its host-side mirror:
a ctypes binding of every entry point plus thin helpers that take torch
tensors for device memory and streams.  The operation names follow the
reference's C++ hot path (tier/tier.cpp): ``dequant`` = dq_launch (294-298),
``gemv`` = gemv_q / gemv<T> (300-306, 2261-2268), ``linear`` / ``linear_dx`` /
``linear_dx_acc`` = the linear operators (1202-1238), ``lmhead_*`` = the
chunked LM-head loops (3184-3266).

There is no CPU fallback: if libtierk.so is missing or fails to load, importing
the binding raises.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libtierk.so"

# status codes (tk_status)
TK_OK, TK_ERR_INVALID, TK_ERR_UNSUPPORTED, TK_ERR_CUDA, TK_ERR_NOMEM, TK_ERR_TIMEOUT, TK_ERR_DEVICE = range(7)
# block types = the reference's QT_* codes (tier/quant.h:20-23)
F32, F16, Q4_0, Q4_1, Q5_0, Q5_1, Q8_0 = 0, 1, 2, 3, 6, 7, 8
Q2_K, Q3_K, Q4_K, Q5_K, Q6_K, BF16, F16X2 = 10, 11, 12, 13, 14, 30, 100
IQ4_NL, IQ4_XS, TQ1_0, TQ2_0, MXFP4, NF4, FP4 = 20, 23, 34, 35, 39, 200, 201
# lattice types: decode after Context.set_iq_grids
IQ2_XXS, IQ2_XS, IQ3_XXS, IQ1_S, IQ3_S, IQ2_S, IQ1_M = 16, 17, 18, 19, 21, 22, 29
QTYPES = {"F32": F32, "F16": F16, "BF16": BF16, "Q4_0": Q4_0, "Q4_1": Q4_1, "Q5_0": Q5_0, "Q5_1": Q5_1,
          "Q8_0": Q8_0, "Q2_K": Q2_K, "Q3_K": Q3_K, "Q4_K": Q4_K, "Q5_K": Q5_K, "Q6_K": Q6_K,
          "IQ4_NL": IQ4_NL, "IQ4_XS": IQ4_XS, "TQ1_0": TQ1_0, "TQ2_0": TQ2_0, "MXFP4": MXFP4, "NF4": NF4, "FP4": FP4,
          "IQ2_XXS": IQ2_XXS, "IQ2_XS": IQ2_XS, "IQ2_S": IQ2_S, "IQ3_XXS": IQ3_XXS, "IQ3_S": IQ3_S, "IQ1_S": IQ1_S,
          "IQ1_M": IQ1_M}
BLOCK = {F32: (1, 4), F16: (1, 2), BF16: (1, 2), Q4_0: (32, 18), Q4_1: (32, 20), Q5_0: (32, 22), Q5_1: (32, 24),
         Q8_0: (32, 34), Q2_K: (256, 84), Q3_K: (256, 110), Q4_K: (256, 144), Q5_K: (256, 176), Q6_K: (256, 210),
         IQ4_NL: (32, 18), IQ4_XS: (256, 136), TQ1_0: (256, 54), TQ2_0: (256, 66), MXFP4: (32, 17),
         NF4: (64, 36), FP4: (64, 36),
         IQ2_XXS: (256, 66), IQ2_XS: (256, 74), IQ2_S: (256, 82), IQ3_XXS: (256, 98), IQ3_S: (256, 110),
         IQ1_S: (256, 50), IQ1_M: (256, 56)}
# activation dtypes
DT_F32, DT_F16, DT_BF16 = 0, 1, 2
# product sets
X3_AUTO, X3_REF, X3_HHL, X2, X1 = 0, 1, 2, 3, 4
QFUSED = 0x100   # OR into `products`: decode a quantized W inside the GEMM
IPC_HANDLE_BYTES = 64   # TK_IPC_HANDLE_BYTES
WFROZEN = 0x200  # OR into tk_gemv's qtype: W is never written by earlier kernels (early weight fetch)
WREUSE = 0x400   # OR into linear products: reuse the previous call's fp16 expansion of the same (unchanged) W
# kernel families for profiling
PROF_GEMM, PROF_DEQUANT, PROF_SPLIT, PROF_GEMV, PROF_LMHEAD, PROF_COMM = range(6)


class TierkError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"tierk status {status}: {msg}")
        self.status = status


class Weight(ctypes.Structure):
    """tk_weight: a frozen W[rows, cols] resident on the device."""
    _fields_ = [("qtype", ctypes.c_int), ("rows", ctypes.c_int), ("cols", ctypes.c_int),
                ("scale_log2", ctypes.c_int), ("row_bytes", ctypes.c_size_t), ("data", ctypes.c_void_p)]


class IqGrids(ctypes.Structure):
    """tk_iq_grids: host pointers to the six lattice tables (int8)."""
    _fields_ = [(n, ctypes.c_void_p) for n in ("iq2xxs", "iq2xs", "iq2s", "iq3xxs", "iq3s", "iq1s")]


# (name, rows, cols) of each table, in tk_iq_grids order
IQ_GRID_SHAPES = [("iq2xxs", 256, 8), ("iq2xs", 512, 8), ("iq2s", 1024, 8), ("iq3xxs", 256, 4), ("iq3s", 512, 4),
                  ("iq1s", 2048, 8)]


def iq_grids_from_gguf() -> dict:
    """The lattice tables as int8 arrays, taken from gguf-py's IQ*.grid (the
    numbers of tier/quant_tables.h).  Needs the gguf package."""
    import numpy as np
    from gguf import quants
    out = {}
    for (name, rows, cols), cls in zip(IQ_GRID_SHAPES, ("IQ2_XXS", "IQ2_XS", "IQ2_S", "IQ3_XXS", "IQ3_S", "IQ1_S")):
        q = getattr(quants, cls)
        q.init_grid()
        g = np.asarray(q.grid, dtype=np.float64).reshape(rows, cols)
        out[name] = np.ascontiguousarray(g.astype(np.int8))
    return out


_P = ctypes.c_void_p
_I = ctypes.c_int
_SZ = ctypes.c_size_t
_F = ctypes.c_float

# (name, restype, argtypes) -- mirrors include/tierk.h
SIGNATURES = [
    ("tk_init", _I, [_I, ctypes.POINTER(_P)]),
    ("tk_destroy", None, [_P]),
    ("tk_last_error_string", ctypes.c_char_p, []),
    ("tk_reserve", _I, [_P, _SZ]),
    ("tk_workspace_bytes", _SZ, [_P]),
    ("tk_sync_status", _I, [_P, _P]),
    ("tk_launch_count", ctypes.c_uint64, [_P]),
    ("tk_profile", _I, [_P, _I]),
    ("tk_profile_read", _I, [_P, _I, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_uint64)]),
    ("tk_row_bytes", _SZ, [_I, _I]),
    ("tk_set_iq_grids", _I, [_P, ctypes.POINTER(IqGrids)]),
    ("tk_lmhead_chunk", _I, [_SZ, _I, _I, _I]),
    ("tk_dequant", _I, [_P, _I, _P, _SZ, _I, _I, _I, _I, _P, _P]),
    ("tk_gemv", _I, [_P, _I, _P, _SZ, _I, _I, _P, _I, _I, _P, _I, _P]),
    ("tk_gemv_multi", _I, [_P, _I, _I, _P, _P, _P, _P, _SZ, _I, _P, _I, _I, _P]),
    ("tk_linear_fwd", _I, [_P, ctypes.POINTER(Weight), _P, _I, _I, _I, _P, _I, _F, _I, _P]),
    ("tk_linear_dx", _I, [_P, ctypes.POINTER(Weight), _P, _I, _I, _I, _P, _I, _F, _I, _P]),
    ("tk_linear_fwd_noalloc", _I, [_P, ctypes.POINTER(Weight), _P, _I, _I, _I, _P, _I, _F, _I, _P]),
    ("tk_weight_split_f32", _I, [_P, _P, _I, _I, _P, ctypes.POINTER(_I), _P]),
    ("tk_split3", _I, [_P, _P, _SZ, _P, _P, _P, _P]),
    ("tk_quantize", _I, [_P, _I, _P, _I, _I, _I, _I, _P, _SZ, _P]),
    ("tk_tq_open", _I, [ctypes.c_char_p, ctypes.POINTER(_P)]),
    ("tk_tq_close", None, [_P]),
    ("tk_tq_count", _I, [_P]),
    ("tk_tq_find", _I, [_P, ctypes.c_char_p]),
    ("tk_tq_entry", _I, [_P, _I, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(_I), ctypes.POINTER(_I),
                         ctypes.POINTER(_I), ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64),
                         ctypes.POINTER(ctypes.c_double)]),
    ("tk_tq_read", _I, [_P, _I, _P, _I, _P]),
    ("tk_tq_write", _I, [ctypes.c_char_p, _I, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(_I),
                         ctypes.POINTER(_I), ctypes.POINTER(_I), ctypes.POINTER(_P), ctypes.POINTER(ctypes.c_double),
                         ctypes.c_char_p]),
    ("tk_qtype_from_name", _I, [ctypes.c_char_p]),
    ("tk_qtype_name", ctypes.c_char_p, [_I]),
    ("tk_comm_init", _I, [_P, _I, _I, _SZ, _P]),
    ("tk_comm_connect", _I, [_P, _P]),
    ("tk_linear_dx_rs", _I, [_P, ctypes.POINTER(Weight), _P, _I, _I, _I, _P, _I, _I, _P]),
    ("tk_linear_fwd_dx", _I, [_P, ctypes.POINTER(Weight), _P, _I, _I, _I, _P, _I, _P, _I, _I, _I, _P, _I, _I, _P]),
    ("tk_linear_fwd_dx_rs", _I, [_P, ctypes.POINTER(Weight), _P, _I, _I, _I, _P, _I, _P, _I, _I, _I, _P, _I, _I,
                                 _P]),
    ("tk_allgather", _I, [_P, _P, _SZ, _P, _P]),
    ("tk_allreduce_f32", _I, [_P, _P, _SZ, _P]),
    ("tk_reshard_cols", _I, [_P, _P, _I, _I, _SZ, _I, _P, _SZ, _P]),
    ("tk_reshard_cols_send", _I, [_P, _P, _I, _I, _SZ, _I, _P]),
    ("tk_reshard_cols_recv", _I, [_P, _P, _SZ, _I, _P]),
    ("tk_lmhead_merge", _I, [_P, _I, _P, _P, _P, _P, _P, _I, _P]),
    ("tk_lmhead_stats", _I, [_P, _P, _I, _I, _I, _P, _I, _P, _P, _F, _I, _I, _P, _P, _P, _P, _P]),
    ("tk_lmhead_grad", _I, [_P, _P, _I, _I, _I, _P, _I, _P, _P, _I, _F, _I, _I, _P, _P, _P, _P]),
    ("tk_lmhead_loss", _I, [_P, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    ("tk_lmhead_rescale", _I, [_P, _I, _P, _P, _P, _P, _I, _P]),
    ("tk_lmhead_fused", _I, [_P, _P, _I, _I, _I, _P, _I, _P, _P, _F, _I, _I, _P, _P, _P, _P, _P, _P]),
    ("tk_lmhead_finish", _I, [_P, _P, _I, _I, _I, _I, _P, _P, _I, _F, _P, _P, _P, _P]),
]

_lib = None


def load(path: str | os.PathLike | None = None) -> ctypes.CDLL:
    """Load libtierk.so (raises if absent -- there is no fallback)."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise RuntimeError(f"libtierk.so not built ({p}); run `python -m tier_b200.build`")
    lib = ctypes.CDLL(str(p))
    for name, res, args in SIGNATURES:
        f = getattr(lib, name)
        f.restype = res
        f.argtypes = args
    if path is None:
        _lib = lib
    return lib


def row_bytes(qtype: int, cols: int) -> int:
    be, bb = BLOCK[qtype]
    return cols // be * bb


def lmhead_chunk(device_bytes: int, hidden: int, seq: int, vocab: int) -> int:
    """tk_lmhead_chunk: the reference's lm_chunk rule (tier/tier.cpp:2015-2017)
    with chunks in multiples of 256; device_bytes is the GPU's total memory."""
    return int(load().tk_lmhead_chunk(device_bytes, hidden, seq, vocab))


def _check(st: int):
    if st != TK_OK:
        raise TierkError(st, load().tk_last_error_string().decode())


def _ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(stream) -> int | None:
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    return getattr(stream, "cuda_stream", stream)


class Context:
    """A tk_ctx bound to one CUDA device."""

    def __init__(self, device: int = 0):
        self.lib = load()
        h = _P()
        _check(self.lib.tk_init(device, ctypes.byref(h)))
        self.h = h
        self.device = device
        self.peers = None        # (rank, world) once host.connect_peers has set up the peer buffers

    def close(self):
        if self.h:
            self.lib.tk_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- diagnostics ----
    def launches(self) -> int:
        return int(self.lib.tk_launch_count(self.h))

    def sync_status(self, stream=None):
        _check(self.lib.tk_sync_status(self.h, _stream(stream)))

    def profile(self, enable: bool, resume: bool = False):
        """Start a new per-launch timing record (enable), resume the current
        one (enable and resume), or pause it (not enable; the record is kept)."""
        _check(self.lib.tk_profile(self.h, (2 if resume else 1) if enable else 0))

    def profile_read(self, kind: int) -> tuple[float, int]:
        t = ctypes.c_double(0)
        n = ctypes.c_uint64(0)
        _check(self.lib.tk_profile_read(self.h, kind, ctypes.byref(t), ctypes.byref(n)))
        return t.value, int(n.value)

    def reserve(self, nbytes: int):
        _check(self.lib.tk_reserve(self.h, nbytes))

    # ---- operations (torch tensors in, device pointers to the C ABI) ----
    def set_iq_grids(self, grids: dict | None = None):
        """Register the IQ1/IQ2/IQ3 lattice tables (tk_set_iq_grids): a dict of
        int8 arrays keyed as IQ_GRID_SHAPES, or None for iq_grids_from_gguf()."""
        import numpy as np
        grids = iq_grids_from_gguf() if grids is None else grids
        keep = []
        s = IqGrids()
        for name, rows, cols in IQ_GRID_SHAPES:
            a = np.ascontiguousarray(grids[name], dtype=np.int8)
            if a.shape != (rows, cols):
                raise ValueError(f"{name}: expected shape {(rows, cols)}, got {a.shape}")
            keep.append(a)
            setattr(s, name, a.ctypes.data)
        _check(self.lib.tk_set_iq_grids(self.h, ctypes.byref(s)))

    def dequant(self, qtype, blocks, rows, cols, out, r0=0, out_dtype=DT_F32, row_bytes_=None, stream=None):
        rb = row_bytes_ if row_bytes_ is not None else row_bytes(qtype, cols)
        _check(self.lib.tk_dequant(self.h, qtype, _ptr(blocks), rb, r0, rows, cols, out_dtype, _ptr(out),
                                   _stream(stream)))
        return out

    def gemv(self, qtype, W, N, K, x, y, M=1, ldx=None, ldy=None, row_bytes_=None, stream=None):
        rb = row_bytes_ if row_bytes_ is not None else row_bytes(qtype & ~WFROZEN, K)
        _check(self.lib.tk_gemv(self.h, qtype, _ptr(W), rb, N, K, _ptr(x), ldx or K, M, _ptr(y), ldy or N,
                                _stream(stream)))
        return y

    def gemv_multi(self, qtype, Ws, rows, ys, K, x, M=1, ldx=None, row_bytes_=None, stream=None):
        """ys[i][:M, :rows[i]] = x . Ws[i]^T for weights that share x (tk_gemv_multi):
        one launch for a layer's q/k/v or gate/up."""
        n = len(Ws)
        rb = row_bytes_ if row_bytes_ is not None else row_bytes(qtype & ~WFROZEN, K)
        wp = (ctypes.c_void_p * n)(*[w.data_ptr() for w in Ws])
        rp = (ctypes.c_int * n)(*rows)
        yp = (ctypes.c_void_p * n)(*[y.data_ptr() for y in ys])
        lp = (ctypes.c_int * n)(*[y.stride(0) for y in ys])
        _check(self.lib.tk_gemv_multi(self.h, qtype, n, wp, rp, yp, lp, rb, K, _ptr(x), ldx or K, M,
                                      _stream(stream)))
        return ys

    def linear(self, W: Weight, X, M, Y, x_dtype=DT_F32, ldx=None, ldy=None, beta=0.0, products=X3_AUTO,
               stream=None):
        _check(self.lib.tk_linear_fwd(self.h, ctypes.byref(W), _ptr(X), x_dtype, M, ldx or W.cols, _ptr(Y),
                                      ldy or W.rows, beta, products, _stream(stream)))
        return Y

    def linear_dx(self, W: Weight, dY, M, dX, dy_dtype=DT_F32, lddy=None, lddx=None, beta=0.0, products=X3_AUTO,
                  stream=None):
        _check(self.lib.tk_linear_dx(self.h, ctypes.byref(W), _ptr(dY), dy_dtype, M, lddy or W.rows, _ptr(dX),
                                     lddx or W.cols, beta, products, _stream(stream)))
        return dX

    def linear_dx_acc(self, W: Weight, dY, M, dX, **kw):
        return self.linear_dx(W, dY, M, dX, beta=1.0, **kw)

    def linear_fwd_dx(self, W: Weight, X, Mx, Y, dY, Md, dX, x_dtype=DT_F32, dy_dtype=None, ldx=None, ldy=None,
                      lddy=None, lddx=None, products=X3_AUTO, stream=None):
        """Y = X . W^T and dX = dY . W in one launch (tk_linear_fwd_dx)."""
        dy_dtype = x_dtype if dy_dtype is None else dy_dtype
        _check(self.lib.tk_linear_fwd_dx(self.h, ctypes.byref(W), _ptr(X), x_dtype, Mx, ldx or W.cols, _ptr(Y),
                                         ldy or W.rows, _ptr(dY), dy_dtype, Md, lddy or W.rows, _ptr(dX),
                                         lddx or W.cols, products, _stream(stream)))
        return Y, dX

    def quantize(self, qtype, x, rows, cols, out, x_dtype=DT_F32, ldx=None, row_bytes_=None, stream=None):
        """out (uint8 [rows, row_bytes]) = x quantized to qtype, byte-exact with the reference's q_row."""
        rb = row_bytes_ if row_bytes_ is not None else row_bytes(qtype, cols)
        _check(self.lib.tk_quantize(self.h, qtype, _ptr(x), x_dtype, rows, cols, ldx or cols, _ptr(out), rb,
                                    _stream(stream)))
        return out

    # ---- reduce-scatter over peer memory (multi-GPU) ----
    def comm_init(self, rank: int, world: int, recv_bytes: int) -> bytes:
        """Allocate this rank's receive buffer; returns its IPC handle (64 bytes)."""
        buf = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
        _check(self.lib.tk_comm_init(self.h, rank, world, recv_bytes, buf))
        return buf.raw

    def comm_connect(self, handles: bytes):
        """Open the peers' buffers: `handles` = every rank's handle, in rank order."""
        buf = ctypes.create_string_buffer(handles, len(handles))
        _check(self.lib.tk_comm_connect(self.h, buf))

    def linear_dx_rs(self, W: Weight, dY, M, dX_rows, dy_dtype=DT_F32, lddy=None, ldd=None, products=X3_AUTO,
                     stream=None):
        """This rank's token rows of sum over ranks of dY . W (tk_linear_dx_rs)."""
        _check(self.lib.tk_linear_dx_rs(self.h, ctypes.byref(W), _ptr(dY), dy_dtype, M, lddy or W.rows, _ptr(dX_rows),
                                        ldd or W.cols, products, _stream(stream)))
        return dX_rows

    def linear_fwd_dx_rs(self, W: Weight, X, Mx, Y, dY, Md, dX_rows, x_dtype=DT_F32, dy_dtype=None, ldx=None,
                         ldy=None, lddy=None, ldd=None, products=X3_AUTO, stream=None):
        """Y = X . W^T (this rank's columns) and this rank's token rows of the
        summed dY . W, in one launch (tk_linear_fwd_dx_rs)."""
        dy_dtype = x_dtype if dy_dtype is None else dy_dtype
        _check(self.lib.tk_linear_fwd_dx_rs(self.h, ctypes.byref(W), _ptr(X), x_dtype, Mx, ldx or W.cols, _ptr(Y),
                                            ldy or W.rows, _ptr(dY), dy_dtype, Md, lddy or W.rows, _ptr(dX_rows),
                                            ldd or W.cols, products, _stream(stream)))
        return Y, dX_rows

    def allgather(self, src, dst, nbytes=None, stream=None):
        """dst = every rank's src in rank order (tk_allgather)."""
        nb = nbytes if nbytes is not None else src.numel() * src.element_size()
        _check(self.lib.tk_allgather(self.h, _ptr(src), nb, _ptr(dst), _stream(stream)))
        return dst

    def reshard_cols(self, src, dst, stream=None):
        """Column shards src [M, n] -> row shard dst [M/world, world*n] (tk_reshard_cols)."""
        M, n = src.shape
        _check(self.lib.tk_reshard_cols(self.h, _ptr(src), M, n, src.stride(0), src.element_size(), _ptr(dst),
                                        dst.stride(0), _stream(stream)))
        return dst

    def reshard_cols_send(self, src, stream=None):
        M, n = src.shape
        _check(self.lib.tk_reshard_cols_send(self.h, _ptr(src), M, n, src.stride(0), src.element_size(),
                                             _stream(stream)))

    def reshard_cols_recv(self, dst, stream=None):
        _check(self.lib.tk_reshard_cols_recv(self.h, _ptr(dst), dst.stride(0), dst.element_size(), _stream(stream)))
        return dst

    def allreduce_f32(self, buf, stream=None):
        """buf = sum over ranks, in rank order (tk_allreduce_f32)."""
        _check(self.lib.tk_allreduce_f32(self.h, _ptr(buf), buf.numel(), _stream(stream)))
        return buf

    def lmhead_merge(self, n, rmax, rsum, amax, tgt, dX=None, H=0, stream=None):
        """Merge the vocabulary shards' running LM-head state (tk_lmhead_merge)."""
        _check(self.lib.tk_lmhead_merge(self.h, n, _ptr(rmax), _ptr(rsum), _ptr(amax), _ptr(tgt), _ptr(dX), H,
                                        _stream(stream)))

    def weight_split_f32(self, W32, rows, cols, planes, stream=None) -> int:
        sc = _I(0)
        _check(self.lib.tk_weight_split_f32(self.h, _ptr(W32), rows, cols, _ptr(planes), ctypes.byref(sc),
                                            _stream(stream)))
        return sc.value

    def split3(self, x, h, m, l, stream=None):
        _check(self.lib.tk_split3(self.h, _ptr(x), x.numel(), _ptr(h), _ptr(m), _ptr(l), _stream(stream)))

    def lmhead_stats(self, W, v0, V_shard, H, X, T, labels, mask, softcap, chunk, rmax, rsum, amax, tgt,
                     products=X3_REF, stream=None):
        _check(self.lib.tk_lmhead_stats(self.h, _ptr(W), v0, V_shard, H, _ptr(X), T, _ptr(labels), _ptr(mask),
                                        softcap, chunk, products, _ptr(rmax), _ptr(rsum), _ptr(amax), _ptr(tgt),
                                        _stream(stream)))

    def lmhead_grad(self, W, v0, V_shard, H, X, T, labels, mask, n_loss, softcap, chunk, rmax, rsum, dX,
                    products=X3_REF, stream=None):
        _check(self.lib.tk_lmhead_grad(self.h, _ptr(W), v0, V_shard, H, _ptr(X), T, _ptr(labels), _ptr(mask),
                                       n_loss, softcap, chunk, products, _ptr(rmax), _ptr(rsum), _ptr(dX),
                                       _stream(stream)))

    def lmhead_loss(self, T, labels, mask, rmax, rsum, amax, tgt, loss, hits, stream=None):
        _check(self.lib.tk_lmhead_loss(self.h, T, _ptr(labels), _ptr(mask), _ptr(rmax), _ptr(rsum), _ptr(amax),
                                       _ptr(tgt), _ptr(loss), _ptr(hits), _stream(stream)))

    def lmhead_rescale(self, n, rmax_local, rsum_local, rmax_global, dX=None, H=0, stream=None):
        _check(self.lib.tk_lmhead_rescale(self.h, n, _ptr(rmax_local), _ptr(rsum_local), _ptr(rmax_global),
                                          _ptr(dX) if dX is not None else None, H, _stream(stream)))

    def lmhead_fused(self, W, v0, V_shard, H, X, T, labels, mask, softcap, chunk, rmax, rsum, amax, tgt, dX,
                     products=X3_REF, stream=None):
        _check(self.lib.tk_lmhead_fused(self.h, _ptr(W), v0, V_shard, H, _ptr(X), T, _ptr(labels), _ptr(mask),
                                        softcap, chunk, products, _ptr(rmax), _ptr(rsum), _ptr(amax), _ptr(tgt),
                                        _ptr(dX), _stream(stream)))

    def lmhead_finish(self, W, v0, V_shard, H, T, labels, mask, n_loss, softcap, rsum, tgt, dX, stream=None):
        _check(self.lib.tk_lmhead_finish(self.h, _ptr(W), v0, V_shard, H, T, _ptr(labels), _ptr(mask), n_loss,
                                         softcap, _ptr(rsum), _ptr(tgt), _ptr(dX), _stream(stream)))


def make_weight(qtype: int, rows: int, cols: int, data, scale_log2: int = 0) -> Weight:
    """Describe a device weight tensor (uint8 blocks or fp16 planes) for the C ABI."""
    rb = cols * 2 if qtype in (F16, F16X2) else row_bytes(qtype, cols)
    w = Weight(qtype, rows, cols, scale_log2, rb, data.data_ptr())
    w._owner = data   # the descriptor keeps its device memory alive
    return w


from .host import LinearPath, LMHead  # noqa: E402  (host-side mirror of the reference's operators)

__all__ = ["Context", "Weight", "make_weight", "load", "row_bytes", "lmhead_chunk", "IqGrids", "IQ_GRID_SHAPES",
           "iq_grids_from_gguf", "LinearPath", "LMHead", "TierkError"]
