"""Seeded synthetic inputs for the benchmark configurations (numpy default_rng;
generation order fixed here).  No dataset is involved: the reference measures
this path on no public suite, so these stand in with the stated shapes and
value distributions.

  C1 q8_0 GEMV     : per block s = max|N(0,0.02)| over 32 draws, d = fp16(s/127),
                     qs uniform int8 in [-127, 127]; x ~ N(0,1).
  C2 Q4_K GEMM     : d, dmin = fp16(|N(0,0.002)|), 8 sub-scales and 8 mins
                     uniform 0..63 packed as tier/quant.h:47-48 unpacks them,
                     nibbles uniform 0..15; X, dY ~ N(0,1) (bf16 in the bench).
  C3 x3 layer      : W fp32 ~ N(0,0.02), X fp32 ~ N(0,1).
  C4 LM head       : W fp16 ~ N(0,0.02), hidden fp32 ~ N(0,1), labels uniform,
                     mask 1 except the last row.
"""
from __future__ import annotations

import numpy as np


def q8_0_blocks(rng, rows, cols):
    nb = rows * cols // 32
    d = np.abs(rng.standard_normal((nb, 32)) * 0.02).max(axis=1) / 127.0
    b = np.zeros((nb, 34), np.uint8)
    b[:, 0:2] = d.astype(np.float16).view(np.uint8).reshape(nb, 2)
    b[:, 2:] = rng.integers(-127, 128, size=(nb, 32), dtype=np.int16).astype(np.int8).view(np.uint8)
    return b.reshape(rows, -1)


def pack_k_scales(sc, mn):
    """Inverse of q4k_scale_min (tier/quant.h:47-48): 8 scales + 8 mins (6 bits) -> 12 bytes."""
    n = sc.shape[0]
    out = np.zeros((n, 12), np.uint8)
    for j in range(4):
        out[:, j] = (sc[:, j] & 63) | ((sc[:, j + 4] >> 4) << 6)
        out[:, j + 4] = (mn[:, j] & 63) | ((mn[:, j + 4] >> 4) << 6)
        out[:, j + 8] = (sc[:, j + 4] & 15) | ((mn[:, j + 4] & 15) << 4)
    return out


def q4_k_blocks(rng, rows, cols):
    nb = rows * cols // 256
    b = np.zeros((nb, 144), np.uint8)
    b[:, 0:2] = np.abs(rng.standard_normal(nb) * 0.002).astype(np.float16).view(np.uint8).reshape(nb, 2)
    b[:, 2:4] = np.abs(rng.standard_normal(nb) * 0.002).astype(np.float16).view(np.uint8).reshape(nb, 2)
    sc = rng.integers(0, 64, size=(nb, 8)).astype(np.uint8)
    mn = rng.integers(0, 64, size=(nb, 8)).astype(np.uint8)
    b[:, 4:16] = pack_k_scales(sc, mn)
    b[:, 16:] = rng.integers(0, 256, size=(nb, 128), dtype=np.uint8)
    return b.reshape(rows, -1)


def q5_k_blocks(rng, rows, cols):
    nb = rows * cols // 256
    b = np.zeros((nb, 176), np.uint8)
    b[:, 0:2] = np.abs(rng.standard_normal(nb) * 0.002).astype(np.float16).view(np.uint8).reshape(nb, 2)
    b[:, 2:4] = np.abs(rng.standard_normal(nb) * 0.002).astype(np.float16).view(np.uint8).reshape(nb, 2)
    sc = rng.integers(0, 64, size=(nb, 8)).astype(np.uint8)
    mn = rng.integers(0, 64, size=(nb, 8)).astype(np.uint8)
    b[:, 4:16] = pack_k_scales(sc, mn)
    b[:, 16:] = rng.integers(0, 256, size=(nb, 160), dtype=np.uint8)
    return b.reshape(rows, -1)


def random_blocks(rng, qtype, rows, cols, scale_offsets, block_bytes, block_elems):
    """Random bytes with valid fp16 scale fields (tier/check_quant.py:27-48 style)."""
    nb = rows * cols // block_elems
    b = rng.integers(0, 256, size=(nb, block_bytes), dtype=np.uint8)
    for o in scale_offsets:
        b[:, o:o + 2] = (rng.standard_normal(nb) * 0.02).astype(np.float16).view(np.uint8).reshape(nb, 2)
    return b.reshape(rows, -1)


SCALE_OFFSETS = {2: [0], 3: [0, 2], 6: [0], 7: [0, 2], 8: [0], 10: [80, 82], 11: [108], 12: [0, 2], 13: [0, 2],
                 14: [208], 20: [0], 23: [0], 34: [52], 35: [64], 16: [0], 17: [0], 22: [0], 18: [0], 21: [0],
                 19: [0]}


def iq1_m_blocks(rng, rows, cols):
    """IQ1_M (tier/quant.h:112-115): the fp16 block scale spread over the top
    nibbles of the four scale words (nibble k in word k)."""
    nb = rows * cols // 256
    b = rng.integers(0, 256, size=(nb, 56), dtype=np.uint8)
    h = (rng.standard_normal(nb) * 0.02).astype(np.float16).view(np.uint16)
    sc = b[:, 48:56].copy().view(np.uint16).reshape(nb, 4)
    for k in range(4):
        sc[:, k] = (sc[:, k] & 0x0FFF) | (((h >> (4 * k)) & 0xF) << 12)
    b[:, 48:56] = sc.view(np.uint8).reshape(nb, 8)
    return b.reshape(rows, -1)


def mxfp4_blocks(rng, rows, cols):
    """MXFP4 (tier/quant.h:70-71): E8M0 scale bytes 118..124 (2^-10..2^-4) so
    the products stay well inside fp32 and fp16, random nibbles."""
    nb = rows * cols // 32
    b = rng.integers(0, 256, size=(nb, 17), dtype=np.uint8)
    b[:, 0] = rng.integers(118, 125, size=nb, dtype=np.uint8)
    return b.reshape(rows, -1)


def absmax_blocks(rng, rows, cols):
    """NF4 / FP4 (tier/quant.h:72-73): fp32 absmax per 64 elements, random nibbles."""
    nb = rows * cols // 64
    b = rng.integers(0, 256, size=(nb, 36), dtype=np.uint8)
    b[:, 0:4] = np.abs(rng.standard_normal(nb) * 0.05).astype(np.float32).view(np.uint8).reshape(nb, 4)
    return b.reshape(rows, -1)


def blocks_for(rng, qtype, rows, cols):
    from tier_b200 import BLOCK
    be, bb = BLOCK[qtype]
    if qtype == 8:
        return q8_0_blocks(rng, rows, cols)
    if qtype == 12:
        return q4_k_blocks(rng, rows, cols)
    if qtype == 13:
        return q5_k_blocks(rng, rows, cols)
    if qtype == 1:
        return (rng.standard_normal((rows, cols)) * 0.02).astype(np.float16).view(np.uint8)
    if qtype == 30:
        x = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
        return (x.view(np.uint32) >> 16).astype(np.uint16).view(np.uint8)
    if qtype == 0:
        return (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32).view(np.uint8)
    if qtype == 39:
        return mxfp4_blocks(rng, rows, cols)
    if qtype in (200, 201):
        return absmax_blocks(rng, rows, cols)
    if qtype == 29:
        return iq1_m_blocks(rng, rows, cols)
    return random_blocks(rng, qtype, rows, cols, SCALE_OFFSETS[qtype], bb, be)


def rel_fro(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))
