#!/usr/bin/env python3
"""End-to-end check of the hooked engine: tierlm's own training step run by
the reference engine unchanged (integration/_build/tier_ref) and by the engine with
its linear path on libtierk (integration/_build/tier_tk), on the same tiny model and
tokens; the two step losses must agree.

  prepare   (where the reference tree is, no GPU needed) writes
            integration/_build/tiny/: a random-init 2-layer Llama (hidden 256,
            vocab 2048) saved as bf16 safetensors by transformers, its
            tier_arch.txt written by the reference's own arch.py, and
            seq_len int32 token ids; then builds both engines.
  run       (on a GPU) runs one training step of each engine with --bf3
            (the fp16-x3 linear path the bridge routes) and --log, and
            prints both losses and the hooked engine's count of calls
            routed to libtierk as one JSON line; exit 1 if the losses differ
            by more than the tolerance or no linear or LM-head pass took the
            library path.

The model is random, so its loss is near ln(vocab) and the engine's start-up
check that stops a model it computes wrongly would fire:
TIER_NO_SELFCHECK=1 turns that check off for this synthetic model.

usage: python integration/e2e_tiny.py prepare [REF_DIR]
       python integration/e2e_tiny.py run [--tol 1e-3]
"""
from __future__ import annotations

import json
import os
import re
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "integration"))
from build_patched_tier import OUT_DIR, build, default_ref  # noqa: E402

TINY = OUT_DIR / "tiny"
SEQ = 128
LAYERS = 2


def make_model(out: Path, ref: Path) -> None:
    import numpy as np
    import torch
    from transformers import LlamaConfig, LlamaForCausalLM
    torch.manual_seed(0)
    cfg = LlamaConfig(vocab_size=2048, hidden_size=256, intermediate_size=512, num_hidden_layers=LAYERS,
                      num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=512, rms_norm_eps=1e-6,
                      rope_theta=10000.0, tie_word_embeddings=False, bos_token_id=1, eos_token_id=2)
    LlamaForCausalLM(cfg).to(torch.bfloat16).save_pretrained(str(out), safe_serialization=True)
    r = subprocess.run([sys.executable, str(ref / "arch.py"), str(out)], capture_output=True, text=True)
    if r.returncode != 0 or not (out / "tier_arch.txt").exists():
        raise SystemExit("arch.py did not describe the model:\n" + r.stdout + r.stderr)
    rng = np.random.default_rng(0)
    rng.integers(3, cfg.vocab_size, size=SEQ, dtype=np.int32).tofile(out / "tokens.bin")


def prepare(ref: Path) -> None:
    TINY.mkdir(parents=True, exist_ok=True)
    make_model(TINY, ref)
    build(ref, hooked=False)
    build(ref, hooked=True)
    print(TINY)


PROJ = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")
NORMS = ("input_layernorm", "post_attn_ln", "pre_ffn_ln", "post_ffn_ln", "q_norm", "k_norm")


def write_tier_file(path: Path) -> None:
    """The engine's slice layout (the format load_tier_assignment reads,
    tier/tier.cpp:1411-1433: "name tier n ntr" per slot): every layer
    projection at tier 2, frozen, so the engine stores it as fp16 and runs
    it through the x3 linear path the bridge routes; the norms at tier 1,
    trainable, so the step still updates weights. Without this file the
    engine's device budget covers the whole tiny model and every projection
    is a trainable fp32 matrix, which the bridge leaves to the engine.
    Names the architecture lacks are skipped by the loader."""
    lines = ["# slot tier n ntr"]
    for l in range(LAYERS):
        lines += [f"layer_{l}.{s} 2 0 0" for s in PROJ]
        lines += [f"layer_{l}.{s} 1 0 0" for s in NORMS]
    lines.append("layer_-1.final_norm 1 0 0")
    path.write_text("\n".join(lines) + "\n")


def step_loss(engine: Path, work: Path, timeout: int = 600) -> tuple[float, dict]:
    """One training step on the tiny model: the loss from the step log and,
    for the hooked engine, the bridge's count of calls routed to libtierk."""
    work.mkdir(parents=True, exist_ok=True)
    log = work / "step.log"
    for f in (log, work / "adam.bin", work / "tier1.bin"):
        if f.exists():
            f.unlink()
    write_tier_file(work / "tier_assignment.txt")
    env = dict(os.environ, TIER_NO_SELFCHECK="1", TIERK_BRIDGE_STATS="1")
    cmd = [str(engine), str(TINY / "model.safetensors"), str(TINY / "tokens.bin"), str(SEQ), str(work / "adam.bin"),
           str(work / "tier1.bin"), "1e-5", str(LAYERS), "1", "--bf3", "--log", str(log)]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout, env=env, cwd=str(work))
    (work / "stdout.txt").write_text(r.stdout + "\n--- stderr ---\n" + r.stderr)
    if r.returncode != 0 or not log.exists():
        raise SystemExit(f"{engine.name} failed (rc {r.returncode}); see {work / 'stdout.txt'}")
    m = re.search(r"===== step \d+ .*? loss ([-0-9.eE+]+)", log.read_text())
    if not m:
        raise SystemExit(f"{engine.name}: no step loss in {log}")
    st = re.search(r"libtierk bridge: fwd (\d+) dx (\d+) chat (\d+) lm_stats (\d+) lm_grad (\d+)", r.stderr)
    routed = dict(zip(("fwd", "dx", "chat", "lm_stats", "lm_grad"), map(int, st.groups()))) if st else {}
    return float(m.group(1)), routed


def run(tol: float) -> int:
    ref_loss, _ = step_loss(OUT_DIR / "tier_ref", TINY / "run_ref")
    tk_loss, routed = step_loss(OUT_DIR / "tier_tk", TINY / "run_tk")
    diff = abs(tk_loss - ref_loss)
    # the hooked engine must have taken the library path for the layers'
    # linears and both LM-head passes, not fallen back to the reference's code
    took = all(routed.get(k, 0) > 0 for k in ("fwd", "dx", "lm_stats", "lm_grad"))
    print(json.dumps({"check": "tiny llama, one --bf3 training step", "loss_reference": ref_loss,
                      "loss_libtierk": tk_loss, "abs_diff": diff, "tol": tol, "routed_to_libtierk": routed}))
    return 0 if diff <= tol and took else 1


if __name__ == "__main__":
    if len(sys.argv) > 1 and sys.argv[1] == "prepare":
        prepare(Path(sys.argv[2]) if len(sys.argv) > 2 else default_ref())
    elif len(sys.argv) > 1 and sys.argv[1] == "run":
        tol = float(sys.argv[sys.argv.index("--tol") + 1]) if "--tol" in sys.argv else 1e-3
        sys.exit(run(tol))
    else:
        print(__doc__)
        sys.exit(2)
