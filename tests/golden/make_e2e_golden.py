"""Regenerate tests/golden/e2e_tokens.json: the reference engine's translations
of seeded synthetic sources on the synthetic NLLB-600M-shaped INT8 model.

The reference binaries are the reference's own main.c/loader.c/tensor.c/
encoder.c/decoder.c compiled from its sources by oracle/Makefile (target
ref-main) with MAX_GEN_LEN raised to 36 (32 target tokens, the end-to-end
single-sentence configuration) and 132 (up to 128, the sentence-batched one).

    python tests/golden/make_e2e_golden.py [model path]
"""
from __future__ import annotations

import json
import os
import re
import subprocess
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "bare-metal-nllb_b200"))
from nllb_attn import synth_model as sm  # noqa: E402

OUT = os.path.join(HERE, "e2e_tokens.json")
DEFAULT_MODEL = os.environ.get("NLLB_SYNTH_MODEL", "/tmp/nllb_synth/synth_nllb600m_seed0.safetensors")

# name: (source seed, source tokens between [src_lang] and [2], max_gen)
CASES = {
    "cfg0_seed0": (0, 16, 36),
    "cfg4_len16": (41, 16, 132),
    "cfg4_len40": (42, 40, 132),
    "cfg4_len100": (43, 100, 132),
}
SRC, TGT = "eng_Latn", "fra_Latn"


def run_reference(model: str, src_ids, max_gen: int):
    exe = os.path.join(REPO, "oracle", "_ref", f"pico_nllb_g{max_gen}")
    args = [exe, model, SRC, TGT] + [str(t) for t in src_ids[1:-1]]
    t0 = time.time()
    out = subprocess.run(args, capture_output=True, text=True, check=True).stdout
    dt = time.time() - t0
    toks = [int(t) for t in re.search(r"^tokens:(.*)$", out, re.M).group(1).split()]
    best = re.search(r"^best: (\d+) tokens, score=([-0-9.]+), enc=(\d+)ms, dec=(\d+)ms, ([0-9.]+) tok/s", out, re.M)
    return toks, {"n_out": int(best.group(1)), "score_2dp": float(best.group(2)),
                  "enc_ms": int(best.group(3)), "dec_ms": int(best.group(4)),
                  "tok_s": float(best.group(5)), "wall_s": round(dt, 2)}


def main() -> None:
    model = sys.argv[1] if len(sys.argv) > 1 else DEFAULT_MODEL
    sm.ensure_model(model, seed=0)
    subprocess.run(["make", "-C", os.path.join(REPO, "oracle"), "ref-main"], check=True)
    res = {"model": {"generator": "nllb_attn.synth_model.write_model", "seed": 0},
           "src_lang": SRC, "tgt_lang": TGT, "tgt_lang_id": sm.LANG[TGT], "cases": {}}
    for name, (seed, n, max_gen) in CASES.items():
        src = sm.source_ids(seed, n, SRC)
        toks, info = run_reference(model, src, max_gen)
        res["cases"][name] = {"seed": seed, "n_tokens": n, "max_gen": max_gen, "src": src,
                              "tokens": toks, "reference": info}
        print(name, len(src), "->", len(toks), info)
    with open(OUT, "w") as f:
        json.dump(res, f, indent=1)
    print("wrote", OUT)


if __name__ == "__main__":
    main()
