#!/usr/bin/env python3
"""Generate the committed golden fixtures under tests/golden/.

Run in a container that has the reference tree and gguf-py 0.19.0 (the
reference's own dequant oracle, tier/check_quant.py:5,71); the outputs are small
.npz files that travel with the repository, so the tests never need either.

Sources of truth recorded per fixture:
  dequant_golden.npz   random blocks generated like tier/check_quant.py:27-48
                       (random bytes, valid fp16 scale fields); expected fp32
                       values from gguf-py `quants.dequantize`, cross-checked
                       bit-for-bit against the reference's quant.h q_val built
                       in place (oracle/_ref/libtkref.so), plus the fp16-storage
                       values tier_fp16(q_val) the training path stores
                       (tier/tier.cpp:294-296).  NF4 and FP4 are tierlm's own
                       types (no gguf-py type): their values come from the
                       reference's quant.h alone.
  quantize_golden.npz  reference q_row bytes (tier/quant.h:201-204) for
                       Q8_0/Q4_K/Q5_K/Q6_K on seeded rows; Q8_0 also equals
                       gguf-py's quantizer (tier/check_quant.py:114).
  split3_golden.npz    reference split3_fp_k (tier/tier.cpp:869-870), run
                       from the extracted kernel body, on seeded and edge values.
  dlogit_golden.npz    reference dlogit_kernel (tier/tier.cpp:736-748) on a
                       small seeded chunk, with and without softcap.
  lse_golden.npz       reference lse_chunk_kernel (tier/tier.cpp:750-759), each
                       block run as 256 host threads with a barrier for
                       __syncthreads: running max / Σexp / argmax / target
                       merged into a seeded prior state, with a masked row, an
                       argmax tie and labels on both sides of the chunk.

usage: python tests/golden/gen_golden.py   (from the repository root)
"""
import ctypes
import os
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
HERE = Path(__file__).resolve().parent


def load_ref():
    so = ROOT / "oracle" / "_ref" / "libtkref.so"
    if not so.exists():
        sys.exit("build oracle/_ref first: make -C oracle")
    lib = ctypes.CDLL(str(so))
    lib.ref_q_val.restype = ctypes.c_float
    lib.ref_row_bytes.restype = ctypes.c_size_t
    return lib


P = ctypes.c_void_p


def ptr(a):
    return a.ctypes.data_as(P)


# (type code, gguf name, elems/block, bytes/block, fp16 scale byte offsets)
TYPES = [
    (0, "F32", 1, 4, []),
    (1, "F16", 1, 2, []),
    (30, "BF16", 1, 2, []),
    (2, "Q4_0", 32, 18, [0]),
    (3, "Q4_1", 32, 20, [0, 2]),
    (6, "Q5_0", 32, 22, [0]),
    (7, "Q5_1", 32, 24, [0, 2]),
    (8, "Q8_0", 32, 34, [0]),
    (10, "Q2_K", 256, 84, [80, 82]),
    (11, "Q3_K", 256, 110, [108]),
    (12, "Q4_K", 256, 144, [0, 2]),
    (13, "Q5_K", 256, 176, [0, 2]),
    (14, "Q6_K", 256, 210, [208]),
    # table-level types (tier/quant.h:69-73, 91-93, 116-119); appended so the
    # random stream of the types above is unchanged
    (20, "IQ4_NL", 32, 18, [0]),
    (23, "IQ4_XS", 256, 136, [0]),
    (34, "TQ1_0", 256, 54, [52]),
    (35, "TQ2_0", 256, 66, [64]),
    (39, "MXFP4", 32, 17, []),
    # tierlm's own 64-element types (tier/quant.h:23, 72-73): no gguf-py type,
    # pinned to the reference's quant.h alone; fp32 absmax at byte 0
    (200, "NF4", 64, 36, "f32"),
    (201, "FP4", 64, 36, "f32"),
    # lattice types (tier/quant.h:94-115; tables tier/quant_tables.h)
    (16, "IQ2_XXS", 256, 66, [0]),
    (17, "IQ2_XS", 256, 74, [0]),
    (22, "IQ2_S", 256, 82, [0]),
    (18, "IQ3_XXS", 256, 98, [0]),
    (21, "IQ3_S", 256, 110, [0]),
    (19, "IQ1_S", 256, 50, [0]),
    (29, "IQ1_M", 256, 56, "iq1m"),
]
GGUF_ONLY_REF = {"NF4", "FP4"}
ROWS, COLS = 4, 512


def gen_dequant(ref):
    from gguf import quants, constants
    rng = np.random.default_rng(7)
    out = {}
    for code, name, be, bb, halfs in TYPES:
        gt = getattr(constants.GGMLQuantizationType, name, None)
        if be == 1:
            if name == "F32":
                x = rng.standard_normal(ROWS * COLS).astype(np.float32)
                b = x.view(np.uint8)
            elif name == "F16":
                x = rng.standard_normal(ROWS * COLS).astype(np.float16)
                b = x.view(np.uint8)
            else:
                x = rng.standard_normal(ROWS * COLS).astype(np.float32)
                b = (x.view(np.uint32) >> 16).astype(np.uint16).view(np.uint8)
            b = b.reshape(ROWS, -1).copy()
        else:
            nb = ROWS * COLS // be
            b = rng.integers(0, 256, size=(nb, bb), dtype=np.uint8)
            if halfs == "f32":
                a = np.abs(rng.standard_normal(nb) * 0.05).astype(np.float32).view(np.uint8).reshape(nb, 4)
                b[:, 0:4] = a
            elif halfs == "iq1m":
                # the fp16 block scale lives in the top nibbles of the four
                # scale words (tier/quant.h:113; tier/check_quant.py:40-45)
                h = (rng.standard_normal(nb) * 0.02).astype(np.float16).view(np.uint16)
                sc = b[:, 48:56].copy().view(np.uint16).reshape(nb, 4)
                for k in range(4):
                    sc[:, k] = (sc[:, k] & 0x0FFF) | (((h >> (4 * k)) & 0xF) << 12)
                b[:, 48:56] = sc.view(np.uint8).reshape(nb, 8)
            else:
                for o in halfs:
                    h = (rng.standard_normal(nb) * 0.02).astype(np.float16).view(np.uint8).reshape(nb, 2)
                    b[:, o:o + 2] = h
            b = b.reshape(ROWS, -1).copy()
        rb = ref.ref_row_bytes(code, COLS)
        assert rb == b.shape[1], (name, rb, b.shape)
        got = np.zeros((ROWS, COLS), np.float32)
        ref.ref_dequant(ptr(b), ctypes.c_size_t(rb), code, 0, ROWS, COLS, 0, ptr(got))
        if name in GGUF_ONLY_REF:
            want = got
        else:
            want = quants.dequantize(b.reshape(-1), gt).reshape(ROWS, COLS).astype(np.float32)
            if not np.array_equal(got.view(np.uint32), want.view(np.uint32)):
                sys.exit(f"{name}: reference quant.h disagrees with gguf-py -- not writing fixtures")
        f16 = np.zeros((ROWS, COLS), np.uint16)
        ref.ref_dequant(ptr(b), ctypes.c_size_t(rb), code, 0, ROWS, COLS, 1, ptr(f16))
        out[f"{name}_blocks"] = b
        out[f"{name}_f32"] = want
        out[f"{name}_f16"] = f16
        out[f"{name}_type"] = np.int32(code)
        src = "reference quant.h" if name in GGUF_ONLY_REF else "gguf-py == reference quant.h (bit-exact)"
        print(f"{name:6s} dequant: {src}, {ROWS}x{COLS}")
    np.savez_compressed(HERE / "dequant_golden.npz", **out)


def gen_quantize(ref):
    from gguf import quants, constants
    rng = np.random.default_rng(11)
    x = (rng.standard_normal((4, 1024)) * 0.02).astype(np.float32)
    out = {"x": x}
    for code, name, bb in [(8, "Q8_0", 34), (12, "Q4_K", 144), (13, "Q5_K", 176), (14, "Q6_K", 210)]:
        rb = ref.ref_row_bytes(code, 1024)
        q = np.zeros((4, rb), np.uint8)
        for r in range(4):
            row = np.ascontiguousarray(x[r])
            assert ref.ref_q_row(code, ptr(row), ptr(q[r]), 1024) == 1
        out[f"{name}_bytes"] = q
        if name == "Q8_0":
            g = quants.quantize(x, constants.GGMLQuantizationType.Q8_0).reshape(4, -1)
            assert np.array_equal(g, q), "Q8_0 quantizer bytes differ from gguf-py"
        print(f"{name:6s} quantize: {q.shape[1]} bytes/row")
    np.savez_compressed(HERE / "quantize_golden.npz", **out)


def gen_split3(ref):
    rng = np.random.default_rng(5)
    edge = np.array([0.0, -0.0, 1.0, -1.0, 65504.0, 65520.0, 7e4, -7e4, 6.1e-5, 5.96e-8, 2.98e-8, 1e-10,
                     3.14159265, -2.718281828, 1e-4 + 1e-9, 0.02, 1.0009765625, 2049.0], np.float32)
    x = np.concatenate([edge, rng.standard_normal(4000).astype(np.float32),
                        (rng.standard_normal(2000) * 0.02).astype(np.float32),
                        (rng.standard_normal(1000) * 1e3).astype(np.float32)])
    n = x.size
    h = np.zeros(n, np.uint16)
    m = np.zeros(n, np.uint16)
    lo = np.zeros(n, np.uint16)
    ref.ref_split3_fp16(ptr(x), ptr(h), ptr(m), ptr(lo), ctypes.c_size_t(n))
    np.savez_compressed(HERE / "split3_golden.npz", x=x, h=h, m=m, l=lo)
    print(f"split3: {n} values")


def gen_dlogit(ref):
    rng = np.random.default_rng(9)
    T, vc, v0, V = 6, 64, 128, 512
    out = {}
    for cap in (0.0, 30.0):
        lg = (rng.standard_normal((T, vc)) * 3).astype(np.float32)
        if cap > 0:
            lg = (cap * np.tanh(lg / cap)).astype(np.float32)
        rmax = (lg.max(axis=1).astype(np.float64) + rng.uniform(0, 1, T)).astype(np.float64)
        rsum = rng.uniform(50, 200, T).astype(np.float64)
        labels = rng.integers(v0 - 8, v0 + vc + 8, size=T).astype(np.int32)
        labels[2] = v0 + 5
        mask = np.array([1, 1, 0, 1, 1, 1], np.uint8)
        n_loss = int(mask[:T - 1].sum())
        dl = np.zeros((T, vc), np.float32)
        ref.ref_dlogit(ptr(lg), ptr(rmax), ptr(rsum), ptr(labels), ptr(dl), T, vc, v0, n_loss, ptr(mask),
                       ctypes.c_float(cap))
        k = f"cap{int(cap)}"
        out.update({f"{k}_lg": lg, f"{k}_rmax": rmax, f"{k}_rsum": rsum, f"{k}_labels": labels,
                    f"{k}_mask": mask, f"{k}_dl": dl, f"{k}_meta": np.array([T, vc, v0, n_loss], np.int32)})
    _ = V
    np.savez_compressed(HERE / "dlogit_golden.npz", **out)
    print("dlogit: 2 cases")


def gen_lse(ref):
    rng = np.random.default_rng(13)
    out = {}
    for k, (T, vc, v0) in enumerate(((9, 700, 256), (6, 256, 0), (5, 100, 1024))):
        lg = (rng.standard_normal((T, vc)) * 4).astype(np.float32)
        lg[2, 10] = lg[2, vc - 3] = lg[2].max() + 1.0        # tie: the lower index wins
        tokens = rng.integers(v0 - 40, v0 + vc + 40, size=T).astype(np.int32)
        mask = np.ones(T, np.uint8)
        mask[3] = 0
        rmax = rng.uniform(-1, 3, T - 1)
        rsum = rng.uniform(10, 100, T - 1)
        amax = np.full(T - 1, 7, np.int32)
        tgt = np.full(T - 1, -5.0, np.float32)
        st = {"rmax": rmax, "rsum": rsum, "amax": amax, "tgt": tgt}
        for n, a in st.items():
            out[f"c{k}_{n}0"] = a.copy()
        ref.ref_lse_chunk(ptr(lg), ptr(rmax), ptr(rsum), ptr(amax), ptr(tgt), ptr(tokens), ptr(mask), T - 1, vc, v0)
        out.update({f"c{k}_lg": lg, f"c{k}_tokens": tokens, f"c{k}_mask": mask, f"c{k}_v0": np.int32(v0),
                    f"c{k}_rmax": rmax, f"c{k}_rsum": rsum, f"c{k}_amax": amax, f"c{k}_tgt": tgt})
    np.savez_compressed(HERE / "lse_golden.npz", **out)
    print("lse_chunk: 3 cases")


def main():
    ref = load_ref()
    gen_dequant(ref)
    gen_quantize(ref)
    gen_split3(ref)
    gen_dlogit(ref)
    gen_lse(ref)


if __name__ == "__main__":
    os.chdir(ROOT)
    main()
