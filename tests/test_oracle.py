"""Pin the CPU oracle (oracle/tk_oracle.c) to the reference's own outputs:
gguf-py 0.19.0 dequant (the reference test's oracle) and the reference's
quant.h / tier.cpp kernel bodies compiled in place, as stored in
tests/golden/ by tests/golden/gen_golden.py."""
import numpy as np
import pytest

from conftest import GOLDEN
from gen import pack_k_scales, q4_k_blocks, q8_0_blocks

DQ = np.load(GOLDEN / "dequant_golden.npz")
TYPE_NAMES = sorted({k.rsplit("_", 1)[0] for k in DQ.files if k.endswith("_type")})


@pytest.mark.parametrize("name", TYPE_NAMES)
def test_dequant_fp32_matches_golden(oracle, name):
    b = DQ[f"{name}_blocks"]
    want = DQ[f"{name}_f32"]
    t = int(DQ[f"{name}_type"])
    got = oracle.dequant(b, t, want.shape[0], want.shape[1], 0)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), name


@pytest.mark.parametrize("name", TYPE_NAMES)
def test_dequant_fp16_storage_matches_golden(oracle, name):
    b = DQ[f"{name}_blocks"]
    want = DQ[f"{name}_f16"]
    t = int(DQ[f"{name}_type"])
    got = oracle.dequant(b, t, want.shape[0], want.shape[1], 1)
    assert np.array_equal(got, want), name


def test_fp16_conversion_exhaustive(oracle):
    # every half code round-trips; numpy's float16 is IEEE RNE like tier_fp16
    L = oracle.L
    for h in range(0, 65536, 7):
        f = L.tko_h2f(h)
        want = np.array([h], np.uint16).view(np.float16).astype(np.float32)[0]
        assert (np.isnan(f) and np.isnan(want)) or np.float32(f).view(np.uint32) == want.view(np.uint32)
    rng = np.random.default_rng(3)
    xs = np.concatenate([rng.standard_normal(20000).astype(np.float32) * s for s in (1e-6, 1e-3, 1, 1e3, 7e4)])
    got = np.array([L.tko_f2h(float(x)) for x in xs], np.uint16)
    want = xs.astype(np.float16).view(np.uint16)
    assert np.array_equal(got, want)


def test_split3_matches_reference_kernel(oracle):
    g = np.load(GOLDEN / "split3_golden.npz")
    h, m, l = oracle.split3(g["x"])
    assert np.array_equal(h, g["h"]) and np.array_equal(m, g["m"]) and np.array_equal(l, g["l"])


@pytest.mark.parametrize("cap", [0, 30])
def test_dlogit_matches_reference_kernel(oracle, cap):
    g = np.load(GOLDEN / "dlogit_golden.npz")
    k = f"cap{cap}"
    T, vc, v0, n_loss = (int(v) for v in g[f"{k}_meta"])
    got = oracle.dlogit(g[f"{k}_lg"], g[f"{k}_rmax"], g[f"{k}_rsum"], g[f"{k}_labels"], g[f"{k}_mask"], v0, n_loss,
                        float(cap))
    want = g[f"{k}_dl"]
    # the reference kernel body was compiled on the host; 1 - y*y may contract to an FMA there or not
    np.testing.assert_allclose(got, want, rtol=2e-7, atol=1e-12)


def test_gemv_warp_order_close_to_f64(oracle):
    rng = np.random.default_rng(0)
    N, K = 64, 1024
    b = q8_0_blocks(rng, N, K)
    x = rng.standard_normal(K).astype(np.float32)
    y = oracle.gemv_warp_order(b, 8, N, K, x)
    ref = oracle.qgemm_f64(b, 8, N, K, x[None])[0]
    assert np.abs(y - ref).max() / np.abs(ref).max() < 1e-5


def test_q4k_generator_scale_packing_roundtrip():
    rng = np.random.default_rng(1)
    sc = rng.integers(0, 64, size=(50, 8)).astype(np.uint8)
    mn = rng.integers(0, 64, size=(50, 8)).astype(np.uint8)
    q = pack_k_scales(sc, mn)
    for j in range(8):
        if j < 4:
            s, m = q[:, j] & 63, q[:, j + 4] & 63
        else:
            s = (q[:, j + 4] & 0xF) | ((q[:, j - 4] >> 6) << 4)
            m = (q[:, j + 4] >> 4) | ((q[:, j] >> 6) << 4)
        assert np.array_equal(s, sc[:, j]) and np.array_equal(m, mn[:, j])


def test_lmhead_f64_small_against_numpy(oracle):
    rng = np.random.default_rng(4)
    V, H, T, chunk = 512, 64, 9, 256
    W = (rng.standard_normal((V, H)) * 0.02).astype(np.float16)
    X = rng.standard_normal((T, H)).astype(np.float32)
    labels = rng.integers(0, V, T).astype(np.int32)
    mask = np.ones(T, np.uint8)
    mask[3] = 0
    loss, n_loss, amax, dX, *_ = oracle.lmhead_f64(W.view(np.uint16), X, labels, mask, 0.0, chunk)
    logits = X.astype(np.float64) @ W.astype(np.float64).T
    logits = logits.astype(np.float32).astype(np.float64)
    lse = np.log(np.exp(logits - logits.max(1, keepdims=True)).sum(1)) + logits.max(1)
    rows = [t for t in range(T - 1) if mask[t]]
    want_loss = sum(lse[t] - logits[t, labels[t + 1]] for t in rows)
    assert n_loss == len(rows)
    assert abs(loss - want_loss) / abs(want_loss) < 1e-9
    P = np.exp(logits - lse[:, None])
    G = np.zeros_like(P)
    for t in rows:
        G[t] = P[t]
        G[t, labels[t + 1]] -= 1
    G /= n_loss
    want_dX = G @ W.astype(np.float64)
    assert np.abs(dX - want_dX).max() < 1e-9
    assert all(amax[t] == int(np.argmax(logits[t])) for t in rows)


def test_quantize_golden_decodes_within_reference_limits(oracle):
    g = np.load(GOLDEN / "quantize_golden.npz")
    x = g["x"]
    lim = {"Q8_0": (8, 0.007), "Q4_K": (12, 0.08), "Q5_K": (13, 0.042), "Q6_K": (14, 0.022)}
    for name, (t, limit) in lim.items():
        q = g[f"{name}_bytes"]
        back = oracle.dequant(q, t, x.shape[0], x.shape[1])
        rel = np.sqrt(((back - x) ** 2).sum() / (x ** 2).sum())
        assert rel < limit, (name, rel)   # tier/check_quant.py:117 limits


def test_reference_build_agrees_with_oracle(oracle):
    from oracle.oracle import RefOracle
    if not RefOracle.available():
        pytest.skip("oracle/_ref not built (reference tree absent)")
    ref = RefOracle()
    rng = np.random.default_rng(2)
    for t, gen in [(8, q8_0_blocks), (12, q4_k_blocks)]:
        b = gen(rng, 8, 2048)
        a = oracle.dequant(b, t, 8, 2048)
        r = ref.dequant(b, t, 8, 2048)
        assert np.array_equal(a.view(np.uint32), r.view(np.uint32))


LSE = np.load(GOLDEN / "lse_golden.npz")


@pytest.mark.parametrize("k", [0, 1, 2])
def test_lse_chunk_matches_reference_kernel(oracle, k):
    """The oracle's lse_chunk restates lse_chunk_kernel (tier/tier.cpp:750-759)
    in its order -- 256 thread-strided fp64 partial sums and a halving tree --
    and reproduces the golden outputs of the kernel body run on 256 host
    threads: bit for bit in the running max, Σexp, argmax (ties to the lower
    index) and target logit, a masked row left untouched."""
    c = f"c{k}_"
    state = [LSE[c + n + "0"].copy() for n in ("rmax", "rsum", "amax", "tgt")]
    oracle.lse_chunk(LSE[c + "lg"], *state, LSE[c + "tokens"], LSE[c + "mask"], int(LSE[c + "v0"]))
    for n, got in zip(("rmax", "rsum", "amax", "tgt"), state):
        assert np.array_equal(got.view(np.uint8), LSE[c + n].view(np.uint8)), n
    assert state[2][3] == LSE[c + "amax0"][3]            # mask[3] == 0: row 3 keeps its prior state


def test_lse_chunk_oracle_agrees_with_reference_live(oracle):
    from oracle.oracle import RefOracle
    if not RefOracle.available():
        pytest.skip("oracle/_ref not built (reference tree absent)")
    ref = RefOracle()
    rng = np.random.default_rng(21)
    for T, vc, v0 in ((12, 1333, 0), (4, 7, 300), (3, 4096, 8192)):
        lg = (rng.standard_normal((T, vc)) * 6).astype(np.float32)
        tokens = rng.integers(v0 - 10, v0 + vc + 10, size=T).astype(np.int32)
        mask = (rng.uniform(size=T) > 0.2).astype(np.uint8)
        st = [rng.uniform(-2, 8, T - 1), rng.uniform(1, 50, T - 1), np.full(T - 1, -1, np.int32),
              np.zeros(T - 1, np.float32)]
        a, b = [x.copy() for x in st], [x.copy() for x in st]
        oracle.lse_chunk(lg, *a, tokens, mask, v0)
        ref.lse_chunk(lg, *b, tokens, mask, v0)
        for x, y in zip(a, b):
            assert np.array_equal(x.view(np.uint8), y.view(np.uint8)), (T, vc, v0)
