"""GPU quantizer (tk_quantize) byte-exact with the reference's CPU quantizer
(q_row, tier/quant.h:201-204): against the committed golden bytes
(tests/golden/quantize_golden.npz, made by the reference's quant.h; Q8_0 also
equal to gguf-py's) and, where the reference build travelled with the repo
(oracle/_ref), against q_row itself on inputs that reach every branch of the
searches: normal rows, outliers, all-zero and constant blocks, all-negative
sub-blocks, tiny (fp16-subnormal scales) and large magnitudes, bf16 sources."""
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).parent / "golden" / "quantize_golden.npz"
TYPES = {"Q8_0": 8, "Q4_K": 12, "Q5_K": 13, "Q6_K": 14}


def dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def gpu_quant(ctx, qt, x, x_dtype=None):
    import torch
    import tier_b200 as tk
    rows, cols = x.shape
    out = torch.full((rows, tk.row_bytes(qt, cols)), 0xAB, dtype=torch.uint8, device="cuda")
    xd = x if isinstance(x, torch.Tensor) else dev(x)
    ctx.quantize(qt, xd, rows, cols, out, x_dtype=tk.DT_F32 if x_dtype is None else x_dtype)
    torch.cuda.synchronize()
    ctx.sync_status()
    return out.cpu().numpy()


@pytest.mark.parametrize("name", list(TYPES))
def test_quantize_golden_bytes(ctx, name):
    g = np.load(GOLDEN)
    got = gpu_quant(ctx, TYPES[name], g["x"])
    assert np.array_equal(got, g[f"{name}_bytes"])


def hard_rows(rng, cols):
    rows = [rng.standard_normal(cols).astype(np.float32) * 0.02,
            rng.standard_normal(cols).astype(np.float32)]
    r = rng.standard_normal(cols).astype(np.float32) * 0.02
    r[rng.integers(0, cols, 7)] *= 300.0                          # outliers
    rows.append(r)
    r = rng.standard_normal(cols).astype(np.float32)
    r[:256] = 0.0                                                # an all-zero super-block
    r[256:288] = 0.75                                            # a constant sub-block
    r[288:320] = -np.abs(r[288:320])                             # all-negative sub-block
    rows.append(r)
    rows.append(rng.standard_normal(cols).astype(np.float32) * 1e-7)    # fp16-subnormal scales
    rows.append(rng.standard_normal(cols).astype(np.float32) * 3e4)     # large
    rows.append(np.abs(rng.standard_normal(cols)).astype(np.float32))    # all positive
    rows.append(np.zeros(cols, np.float32))
    return np.stack(rows)


@pytest.mark.parametrize("name", list(TYPES))
def test_quantize_matches_reference_q_row(ctx, oracle, name):
    import sys
    sys.path.insert(0, str(Path(__file__).parents[1]))
    from oracle.oracle import RefOracle
    if not RefOracle.available():
        pytest.skip("reference build (oracle/_ref) not present")
    ref = RefOracle()
    rng = np.random.default_rng(TYPES[name] + 100)
    qt = TYPES[name]
    x = np.concatenate([hard_rows(rng, 2048), rng.standard_normal((56, 2048)).astype(np.float32) * 0.05])
    got = gpu_quant(ctx, qt, x)
    want = np.stack([ref.quantize_row(qt, r) for r in x])
    bad = [i for i in range(len(x)) if not np.array_equal(got[i], want[i])]
    assert not bad, f"rows {bad[:8]} differ"


@pytest.mark.parametrize("name", list(TYPES))
def test_quantize_bf16_source_and_round_trip(ctx, oracle, name):
    """bf16 input widens exactly: same bytes as quantizing the fp32 copy; the
    bytes dequantize (bit-exact dequant) to within the type's usual error."""
    import torch
    import tier_b200 as tk
    qt = TYPES[name]
    rng = np.random.default_rng(7 + qt)
    rows, cols = 300, 4096
    xb = torch.from_numpy(rng.standard_normal((rows, cols)).astype(np.float32) * 0.02).to(torch.bfloat16)
    a = gpu_quant(ctx, qt, xb.cuda(), x_dtype=tk.DT_BF16)
    b = gpu_quant(ctx, qt, xb.float().numpy())
    assert np.array_equal(a, b)
    back = oracle.dequant(a, qt, rows, cols, 0)
    xf = xb.float().numpy().astype(np.float64)
    rel = np.linalg.norm(back - xf) / np.linalg.norm(xf)
    # measured on N(0, 0.02) rows: Q4_K 7.1 %, Q5_K 3.6 %, Q6_K 1.8 % relative RMS
    assert rel < {8: 0.01, 12: 0.09, 13: 0.045, 14: 0.025}[qt], rel


def test_quantize_to_tq_round_trip(ctx, tmp_path):
    """GPU quantizer -> .tq writer -> reader into device memory: the bytes come
    back unchanged, match the golden quantizer bytes, and each matrix's err is
    its relative RMS dequantization error."""
    import torch
    import tier_b200 as tk
    from tier_b200.tq import TQFile, quantize_to_tq
    g = np.load(GOLDEN)
    x = dev(g["x"])
    names = list(TYPES)
    errs = quantize_to_tq(ctx, tmp_path / "m.tq", [(f"w.{n}", x) for n in names], [TYPES[n] for n in names],
                          meta="#from tierlm test\n")
    with TQFile(tmp_path / "m.tq") as f:
        for i, n in enumerate(names):
            e = f.entries[i]
            assert (e.name, e.qtype, e.rows, e.cols) == (f"w.{n}", TYPES[n], 4, 1024)
            back = f.read(i, device="cuda")
            assert np.array_equal(back.cpu().numpy(), g[f"{n}_bytes"])
            deq = torch.empty(4, 1024, device="cuda")
            ctx.dequant(TYPES[n], back, 4, 1024, deq)
            want = float(np.sqrt(((deq.cpu().numpy().astype(np.float64) - g["x"]) ** 2).sum() / (g["x"].astype(np.float64) ** 2).sum()))
            assert abs(e.err - want) < 1e-6 and abs(errs[i] - want) < 1e-9
