"""`.tq` quantized-base files and the quantization recipes, over libtierk.

Mirrors the reference's file handling: the reader is tq_load
(tier/tier.cpp:274-292), the writer the layout of quant_main
(tier/tier.cpp:2698-2746) and write_tq (tier/quant.py:60-105), and
`recipe_types` restates quant_main's per-matrix type rules.  Quantization
runs on the GPU (tk_quantize, byte-exact with the reference's q_row).
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

from . import Q4_K, Q5_K, Q6_K, Q8_0, _check, load, row_bytes

SLOTS = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


@dataclass
class Entry:
    name: str
    qtype: int
    rows: int
    cols: int
    offset: int
    bytes: int
    err: float


class TQFile:
    """An open `.tq` file: `entries` in file order, `read` to host or device."""

    def __init__(self, path: str):
        self.lib = load()
        h = ctypes.c_void_p()
        _check(self.lib.tk_tq_open(str(path).encode(), ctypes.byref(h)))
        self.h = h
        self.entries = []
        for i in range(self.lib.tk_tq_count(h)):
            nm = ctypes.c_char_p()
            qt, r, c = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
            off, sz, err = ctypes.c_uint64(), ctypes.c_uint64(), ctypes.c_double()
            _check(self.lib.tk_tq_entry(h, i, ctypes.byref(nm), ctypes.byref(qt), ctypes.byref(r), ctypes.byref(c),
                                        ctypes.byref(off), ctypes.byref(sz), ctypes.byref(err)))
            self.entries.append(Entry(nm.value.decode(), qt.value, r.value, c.value, off.value, sz.value, err.value))

    def index(self, name: str) -> int:
        i = self.lib.tk_tq_find(self.h, name.encode())
        if i < 0:
            raise KeyError(name)
        return i

    def read(self, key, device=None):
        """Blocks of one matrix as uint8 [rows, row_bytes]: numpy on the host,
        or a torch tensor on `device`."""
        i = key if isinstance(key, int) else self.index(key)
        e = self.entries[i]
        rb = e.bytes // e.rows if e.rows else 0
        if device is None:
            import numpy as np
            out = np.empty((e.rows, rb), np.uint8)
            _check(self.lib.tk_tq_read(self.h, i, out.ctypes.data_as(ctypes.c_void_p), 0, None))
            return out
        import torch
        out = torch.empty((e.rows, rb), dtype=torch.uint8, device=device)
        _check(self.lib.tk_tq_read(self.h, i, ctypes.c_void_p(out.data_ptr()), 1, None))
        return out

    def close(self):
        if self.h:
            self.lib.tk_tq_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def write_tq(path: str, items, meta=None, errs=None):
    """items: (name, qtype, rows, cols, data) with data a host numpy uint8
    array or a device torch tensor of rows * row_bytes bytes; meta: dict
    (written as "#key value" lines) or preformatted text."""
    lib = load()
    n = len(items)
    names = (ctypes.c_char_p * n)(*[it[0].encode() for it in items])
    qts = (ctypes.c_int * n)(*[it[1] for it in items])
    rows = (ctypes.c_int * n)(*[it[2] for it in items])
    cols = (ctypes.c_int * n)(*[it[3] for it in items])
    ptrs = []
    for it in items:
        d = it[4]
        need = row_bytes(it[1], it[3]) * it[2]
        size = d.numel() * d.element_size() if hasattr(d, "data_ptr") else d.nbytes
        if size != need:
            raise ValueError(f"{it[0]}: {size} bytes, {need} expected")
        ptrs.append(d.data_ptr() if hasattr(d, "data_ptr") else d.ctypes.data)
    data = (ctypes.c_void_p * n)(*ptrs)
    e = (ctypes.c_double * n)(*errs) if errs is not None else None
    if isinstance(meta, dict):
        meta = "".join(f"#{k} {v}\n" for k, v in meta.items())
    _check(lib.tk_tq_write(str(path).encode(), n, names, qts, rows, cols, data, e, meta.encode() if meta else None))


def recipe_base(recipe: str) -> int:
    """Base block type of a recipe name (quant_main, tier/tier.cpp:2702)."""
    if recipe == "Q8_0":
        return Q8_0
    if recipe == "Q6_K":
        return Q6_K
    if recipe.startswith("Q5_K"):
        return Q5_K
    if recipe.startswith("Q4_K"):
        return Q4_K
    raise ValueError(f"unknown recipe {recipe}: Q8_0, Q6_K, Q5_K_M, Q5_K_S, Q4_K_M, Q4_K_S")


def _more(i: int, n: int) -> bool:
    # layers that keep more bits in _M recipes (tier/tier.cpp:2708)
    return i < n // 8 or i >= 7 * n // 8 or (i - n // 8) % 3 == 2


def recipe_types(recipe: str, layers):
    """Type per matrix for a recipe, as quant_main assigns them
    (tier/tier.cpp:2704-2712).  `layers`: per layer, the slots present
    (subset of SLOTS, in SLOTS order).  Returns [(layer, slot, qtype)]."""
    base = recipe_base(recipe)
    mm = len(recipe) > 2 and recipe.endswith("_M")
    ms = len(recipe) > 2 and recipe.endswith("_S")
    nl = len(layers)
    nv = sum(1 for slots in layers if "v_proj" in slots)
    out, iv = [], 0
    for l, slots in enumerate(layers):
        for i, slot in enumerate(SLOTS):
            if slot not in slots:
                continue
            t = base
            if i == 2:
                if mm and _more(iv, nv):
                    t = Q6_K
                elif ms and base == Q4_K and iv < 4:
                    t = Q5_K
                iv += 1
            if i == 6:
                if mm and _more(l, nl):
                    t = Q6_K
                elif ms and base == Q4_K and l < nl // 8:
                    t = Q5_K
            out.append((l, slot, t))
    return out


def quantize_to_tq(ctx, path: str, tensors, qtypes, meta: str | None = None):
    """Quantize device tensors (fp32 or bf16, [rows, cols]) on the GPU and
    write them as a `.tq` file.  tensors / qtypes: parallel lists, names taken
    from `tensors` as (name, tensor).  Each matrix's err is the relative RMS
    error of its dequantized values, sqrt(sum (q - x)^2 / sum x^2), as
    quant_main reports it; the file's "#err" line is the same over all."""
    import torch
    from . import DT_BF16, DT_F32
    items, errs, se, sq = [], [], 0.0, 0.0
    for (name, x), qt in zip(tensors, qtypes):
        rows, cols = x.shape
        if x.stride(1) != 1:                 # the quantizer reads rows of cols contiguous elements
            x = x.contiguous()
        blocks = torch.empty(rows, row_bytes(qt, cols), dtype=torch.uint8, device=x.device)
        ctx.quantize(qt, x, rows, cols, blocks, x_dtype=DT_BF16 if x.dtype == torch.bfloat16 else DT_F32,
                     ldx=x.stride(0))
        back = torch.empty(rows, cols, dtype=torch.float32, device=x.device)
        ctx.dequant(qt, blocks, rows, cols, back)
        xf = x.float()
        e = float(((back.double() - xf.double()) ** 2).sum())
        s = float((xf.double() ** 2).sum())
        se, sq = se + e, sq + s
        errs.append(math.sqrt(e / s) if s > 0 else 0.0)
        items.append((name, qt, rows, cols, blocks))
    text = (meta or "") + f"#err {math.sqrt(se / sq) if sq > 0 else 0.0:.6f}\n"
    write_tq(path, items, text, errs)
    return errs


__all__ = ["TQFile", "Entry", "write_tq", "recipe_base", "recipe_types", "quantize_to_tq", "SLOTS"]
