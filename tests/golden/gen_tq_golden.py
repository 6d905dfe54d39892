"""Writes ref_small.tq: a small quantized-base file made by the reference's own
writer (write_tq, tier/quant.py:60-105), run from the reference tree. The
block bytes are seeded random; tests/test_tq.py regenerates them with the same
seed and checks that tier_b200's reader parses the file and that its writer
reproduces it byte for byte.

usage: python tests/golden/gen_tq_golden.py /path/to/reference/tier
"""
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

# (name, type, rows, cols, bytes per (block elements, block bytes))
ITEMS = [("model.layers.0.self_attn.q_proj.weight", "Q8_0", 3, 64, (32, 34)),
         ("model.layers.0.mlp.down_proj.weight", "Q4_K", 2, 512, (256, 144)),
         ("model.layers.1.self_attn.v_proj.weight", "Q6_K", 1, 256, (256, 210)),
         ("lm_head.weight", "F16", 4, 8, (1, 2))]
META = {"from": "test", "src": "0 0"}


def item_bytes(i):
    _, _, rows, cols, (be, bb) = ITEMS[i]
    return np.random.default_rng(100 + i).integers(0, 256, rows * (cols // be) * bb, dtype=np.uint8).tobytes()


def main(ref_tier):
    sys.path.insert(0, str(ref_tier))
    import quant   # the reference's tier/quant.py
    items = [(nm, ty, rows, cols, (lambda i=i: item_bytes(i))) for i, (nm, ty, rows, cols, _) in enumerate(ITEMS)]
    out = HERE / "ref_small.tq"
    quant.write_tq(str(out), items, META)
    print(out, out.stat().st_size)


if __name__ == "__main__":
    if len(sys.argv) < 2 and not os.environ.get("TIER_REF"):
        raise SystemExit("usage: gen_tq_golden.py <reference tier/ directory>  (or set TIER_REF)")
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ["TIER_REF"])
