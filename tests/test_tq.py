"""`.tq` files (host side, no GPU): tier_b200's reader on a file written by
the reference's own writer (tests/golden/ref_small.tq, made by
tests/golden/gen_tq_golden.py with tier/quant.py's write_tq), its writer
reproducing that file byte for byte, the reference's rejections (tq_load,
tier/tier.cpp:274-292), and quant_main's recipe type rules
(tier/tier.cpp:2704-2712)."""
import sys
from pathlib import Path

import numpy as np
import pytest

HERE = Path(__file__).parent
sys.path.insert(0, str(HERE / "golden"))
from gen_tq_golden import ITEMS, META, item_bytes  # noqa: E402

GOLD = HERE / "golden" / "ref_small.tq"


def test_reader_parses_reference_file():
    import tier_b200 as tk
    from tier_b200.tq import TQFile
    with TQFile(GOLD) as f:
        assert [e.name for e in f.entries] == [it[0] for it in ITEMS]
        for i, (e, (nm, ty, rows, cols, _)) in enumerate(zip(f.entries, ITEMS)):
            assert (e.qtype, e.rows, e.cols) == (tk.QTYPES[ty], rows, cols)
            assert e.offset % 4096 == 0 and e.err == -1.0
            assert f.read(i).tobytes() == item_bytes(i)
        assert f.index("lm_head.weight") == 3
        with pytest.raises(KeyError):
            f.index("missing")


def test_writer_reproduces_reference_file(tmp_path):
    import tier_b200 as tk
    from tier_b200.tq import write_tq
    items = []
    for i, (nm, ty, rows, cols, _) in enumerate(ITEMS):
        b = np.frombuffer(item_bytes(i), np.uint8).reshape(rows, -1).copy()
        items.append((nm, tk.QTYPES[ty], rows, cols, b))
    out = tmp_path / "ours.tq"
    write_tq(out, items, META)
    assert out.read_bytes() == GOLD.read_bytes()
    assert not (tmp_path / "ours.tq.part").exists()


def test_writer_err_column_and_type_names(tmp_path):
    import tier_b200 as tk
    from tier_b200.tq import TQFile, write_tq
    b = np.zeros((2, tk.row_bytes(tk.Q5_K, 256)), np.uint8)
    write_tq(tmp_path / "e.tq", [("w", tk.Q5_K, 2, 256, b)], "#from tierlm Q4_K_S\n", errs=[0.0123456])
    with TQFile(tmp_path / "e.tq") as f:
        assert abs(f.entries[0].err - 0.012346) < 1e-9
    lib = tk.load()
    for name, code in tk.QTYPES.items():
        assert lib.tk_qtype_from_name(name.encode()) == code
        assert lib.tk_qtype_name(code).decode() == name
    assert lib.tk_qtype_from_name(b"NF4") == 200 and lib.tk_qtype_from_name(b"XYZ") == -1


@pytest.mark.parametrize("bad", ["magic", "hb", "size", "type", "cols"])
def test_reader_rejects_like_the_reference(tmp_path, bad):
    import tier_b200 as tk
    from tier_b200.tq import TQFile
    h = "TQB1 4096 1\nw Q4_K 2 512 4096 576 -1\n"
    if bad == "magic":
        h = h.replace("TQB1", "TQB2")
    elif bad == "hb":
        h = h.replace("TQB1 4096", "TQB1 32")
    elif bad == "size":
        h = h.replace(" 576 ", " 575 ")
    elif bad == "type":
        h = h.replace("Q4_K", "Q9_Z")
    else:
        h = h.replace(" 512 ", " 500 ")
    p = tmp_path / "bad.tq"
    p.write_bytes(h.encode().ljust(4096, b"\0") + bytes(4096))
    with pytest.raises(tk.TierkError):
        TQFile(p)


def test_reader_skips_comment_and_short_lines(tmp_path):
    from tier_b200.tq import TQFile
    h = "TQB1 4096 1\n#from x\n\nnot a matrix line\nw Q8_0 1 32 4096 34 -1\n"
    p = tmp_path / "ok.tq"
    p.write_bytes(h.encode().ljust(4096, b"\0") + bytes(4096))
    with TQFile(p) as f:
        assert [e.name for e in f.entries] == ["w"]


def test_recipe_types():
    import tier_b200 as tk
    from tier_b200.tq import SLOTS, recipe_types
    layers = [list(SLOTS)] * 40
    t = {(l, s): q for l, s, q in recipe_types("Q4_K_S", layers)}
    assert all(t[(l, "v_proj")] == (tk.Q5_K if l < 4 else tk.Q4_K) for l in range(40))
    assert all(t[(l, "down_proj")] == (tk.Q5_K if l < 5 else tk.Q4_K) for l in range(40))
    assert all(t[(l, s)] == tk.Q4_K for l in range(40) for s in SLOTS if s not in ("v_proj", "down_proj"))
    m = {(l, s): q for l, s, q in recipe_types("Q5_K_M", layers)}
    more = [l < 5 or l >= 35 or (l - 5) % 3 == 2 for l in range(40)]
    assert [m[(l, "down_proj")] == tk.Q6_K for l in range(40)] == more
    assert [m[(l, "v_proj")] == tk.Q6_K for l in range(40)] == more
    assert {q for _, _, q in recipe_types("Q8_0", layers)} == {tk.Q8_0}
    # layers without v_proj do not advance the v counter
    lay = [[s for s in SLOTS if s != "v_proj"] if l % 2 else list(SLOTS) for l in range(16)]
    v = [(l, q) for l, s, q in recipe_types("Q4_K_S", lay) if s == "v_proj"]
    assert [q for _, q in v] == [tk.Q5_K] * 4 + [tk.Q4_K] * 4 and [l for l, _ in v][:4] == [0, 2, 4, 6]
    with pytest.raises(ValueError):
        recipe_types("Q3_K", layers)


def test_every_block_type_round_trips(tmp_path):
    """One matrix of each of the 27 types of tier/quant.h:25-31: the writer
    records its name and the reader returns the same geometry and bytes."""
    import tier_b200 as tk
    from tier_b200.tq import TQFile, write_tq
    rng = np.random.default_rng(27)
    items = []
    for name, code in sorted(tk.QTYPES.items(), key=lambda kv: kv[1]):
        rows, cols = 3, 512
        b = rng.integers(0, 256, size=(rows, tk.row_bytes(code, cols)), dtype=np.uint8)
        items.append((f"m.{name.lower()}", code, rows, cols, b))
    write_tq(tmp_path / "all.tq", items, "#from tierlm test\n")
    with TQFile(tmp_path / "all.tq") as f:
        assert len(f.entries) == 27
        for i, (nm, code, rows, cols, b) in enumerate(items):
            e = f.entries[i]
            assert (e.name, e.qtype, e.rows, e.cols) == (nm, code, rows, cols)
            assert e.offset % 4096 == 0
            assert f.read(i).tobytes() == b.tobytes()
    text = (tmp_path / "all.tq").read_bytes().split(b"\n")
    assert any(b" IQ1_M " in ln for ln in text) and any(b" MXFP4 " in ln for ln in text)
