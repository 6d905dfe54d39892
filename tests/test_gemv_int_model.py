"""The integer decode GEMVs' arithmetic, modelled in numpy on the CPU and held
against the fp64 oracle: x split per (token, 256-element chunk) into three
exact signed-byte planes after a power-of-two scaling, products of integer
quants and planes summed exactly in int64, Q4_K sub-block scales applied in
integers, the min term through the x sums split into two bytes, and the
fp32 scale factors at the end.  This is the scheme of
tier_b200/csrc/tk_gemv6.cu and tk_gemv7.cu; the GPU tests check the kernels
themselves."""
import numpy as np
import pytest

from gen import q4_k_blocks, q8_0_blocks


def planes(x):
    """x [M, K] fp32 -> (p [3, M, K] int64, scale [M, K/256, 3] float64)."""
    M, K = x.shape
    xc = x.reshape(M, K // 256, 256).astype(np.float32)
    mx = np.abs(xc).max(axis=2)
    E = (mx.view(np.uint32) >> 23) & 0xFF
    s = np.where(mx > 0, np.minimum(148 - E.astype(np.int64), 127), 0)
    up = np.ldexp(np.float32(1.0), s).astype(np.float32)
    xi = np.rint(xc * up[:, :, None]).astype(np.int64)          # round half to even, as cvt.rni
    assert np.abs(xi).max() < (1 << 22)
    b2 = ((xi & 0xFF) ^ 0x80) - 0x80                                # low byte, signed
    r1 = (xi - b2) >> 8
    b1 = ((r1 & 0xFF) ^ 0x80) - 0x80
    b0 = (r1 - b1) >> 8
    assert np.array_equal(b0 * 65536 + b1 * 256 + b2, xi)
    assert np.abs(b0).max() <= 64 and np.abs(b1).max() <= 128 and np.abs(b2).max() <= 128
    p = np.stack([b0, b1, b2]).reshape(3, M, K)
    sc = np.stack([np.ldexp(1.0, 16 - 8 * q - s) for q in range(3)], axis=-1)
    return p, sc


def f16(b):
    return b.view(np.float16).astype(np.float64)


def model_q8_0(blocks, N, K, x):
    p, sc = planes(x)
    M = x.shape[0]
    bl = blocks.reshape(N, K // 32, 34)
    d = f16(bl[:, :, 0:2].copy()).reshape(N, K // 32)
    q = bl[:, :, 2:].view(np.int8).astype(np.int64)                  # [N, nb, 32]
    y = np.zeros((M, N))
    for m in range(M):
        for pl in range(3):
            C = np.einsum("nbk,bk->nb", q, p[pl, m].reshape(K // 32, 32))     # exact int64
            # fp32 products of d and the integer sums, per 256-chunk scale
            t = (d.astype(np.float32) * C.astype(np.float32)).astype(np.float64)
            y[m] += (t.reshape(N, K // 256, 8).sum(axis=2) * sc[m, :, pl][None, :]).sum(axis=1)
    return y


def model_q4_k(blocks, N, K, x):
    p, sc = planes(x)
    M = x.shape[0]
    bl = blocks.reshape(N, K // 256, 144)
    d, dmin = f16(bl[:, :, 0:2].copy()).reshape(N, -1), f16(bl[:, :, 2:4].copy()).reshape(N, -1)
    w = bl[:, :, 4:16].astype(np.int64)
    scl = np.zeros((N, K // 256, 8), np.int64)
    mn = np.zeros_like(scl)
    for j in range(4):                                                # tier/quant.h:47-48
        scl[:, :, j] = w[:, :, j] & 63
        mn[:, :, j] = w[:, :, j + 4] & 63
        scl[:, :, j + 4] = (w[:, :, j + 8] & 15) | ((w[:, :, j] >> 6) << 4)
        mn[:, :, j + 4] = (w[:, :, j + 8] >> 4) | ((w[:, :, j + 4] >> 6) << 4)
    qs = bl[:, :, 16:].astype(np.int64).reshape(N, K // 256, 4, 32)
    nib = np.stack([qs & 15, qs >> 4], axis=3).reshape(N, K // 256, 8, 32)   # sub-block 2j: low, 2j+1: high
    y = np.zeros((M, N))
    for m in range(M):
        for pl in range(3):
            xp = p[pl, m].reshape(K // 256, 8, 32)
            C = np.einsum("nsbk,sbk->nsb", nib, xp)                     # per sub-block, exact
            S = xp.sum(axis=2)                                        # x sums, |S| <= 4096
            S_lo, S_hi = S & 127, S >> 7                              # two bytes, S = hi * 128 + lo
            assert np.array_equal(S_hi * 128 + S_lo, S) and np.abs(S_hi).max() <= 32
            I1 = (scl * C).sum(axis=2)                                # int32 range
            I2 = (mn * (S_hi * 128 + S_lo)[None]).sum(axis=2)
            assert np.abs(I1).max() < (1 << 31) and np.abs(I2).max() < (1 << 31)
            v = (d.astype(np.float32) * I1.astype(np.float32) - (dmin.astype(np.float32) * I2.astype(np.float32)))
            y[m] += (v.astype(np.float64) * sc[m, :, pl][None, :]).sum(axis=1)
    return y


@pytest.mark.parametrize("qtype", [8, 12])
@pytest.mark.parametrize("outlier", [False, True])
def test_integer_decode_model_matches_fp64(oracle, qtype, outlier):
    """Chunks of x at very different magnitudes cost nothing (each has its own
    power of two).  Within a chunk every element is kept to 2^-22 of the
    chunk's largest, so one element 37x the rest leaves the others 17 bits and
    the result ~1e-5 relative (the decode tolerance is 2e-3); without such an
    outlier it is ~1e-7."""
    rng = np.random.default_rng(5 + qtype)
    N, K, M = 96, 1024, 2
    b = q8_0_blocks(rng, N, K) if qtype == 8 else q4_k_blocks(rng, N, K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    x[1, :256] *= 1e-6                                                # chunk scales differ by 2^20
    if outlier:
        x[1, 300] = 37.0                                              # one large element in a chunk
    want = oracle.qgemm_f64(b, qtype, N, K, x)
    got = model_q8_0(b, N, K, x) if qtype == 8 else model_q4_k(b, N, K, x)
    err = [np.linalg.norm(got[m] - want[m]) / np.linalg.norm(want[m]) for m in range(M)]
    assert err[0] < 1e-6
    assert err[1] < (5e-5 if outlier else 1e-6)


def test_planes_are_exact_and_bounded():
    rng = np.random.default_rng(3)
    x = (rng.standard_normal((3, 512)) * np.logspace(-30, 30, 512)).astype(np.float32)
    p, sc = planes(x)
    back = (p[0] * 65536.0 + p[1] * 256.0 + p[2]).reshape(3, 2, 256) * np.ldexp(1.0, -16)
    back = back * (sc[:, :, 0][:, :, None] / 1.0)
    rel = np.abs(back.reshape(3, 512) - x) / np.abs(x).reshape(3, 2, 256).max(axis=2).repeat(256, axis=1)
    assert rel.max() <= 2.0 ** -22
