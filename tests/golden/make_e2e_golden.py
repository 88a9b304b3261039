"""Regenerate tests/golden/e2e_tokens.json: the reference engine's translations
of seeded synthetic sources on the synthetic NLLB-600M-shaped INT8 model, with
the reference's own per-step decision margins.

The reference programs are the reference's own main.c/loader.c/tensor.c/
encoder.c/decoder.c compiled from its sources by oracle/Makefile (target
ref-main) with MAX_GEN_LEN raised to 36 (32 target tokens, the end-to-end
single-sentence configuration) and 132 (up to 128, the sentence-batched one).
The _steplog builds add one stderr line per beam-search step with the sorted
candidate scores (oracle/ref_steplog.h); their arithmetic and token output are
those of the plain builds.

For every case the file holds the source ids, the reference's token ids and
`margins`: for each step from 2 on, the smallest gap between consecutive
sorted candidate scores among the first BEAM_SIZE + 1 (main.c:455-484: those
positions decide which candidates survive and in which beam order).  A token
difference is exempt only after a step whose margin is below 1e-4.

Cases: config 0 (one 16-token sentence, 32 target tokens), three hand-picked
config-4-shaped sentences, and the first 128 sentences of the sentence-batched
workload (nllb_attn.synth_model.config4_sources, seed 4), max 128 tokens.

    python tests/golden/make_e2e_golden.py [model path] [--jobs J] [--reuse]

--reuse keeps the cases of the existing file whose inputs (source ids,
max_gen) are unchanged instead of running the reference again for them.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import subprocess
import sys
import time
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "bare-metal-nllb_b200"))
from nllb_attn import synth_model as sm  # noqa: E402

OUT = os.path.join(HERE, "e2e_tokens.json")
BEAM = 4

# name: (source seed, source tokens between [src_lang] and [2], max_gen)
HAND_PICKED = {
    "cfg0_seed0": (0, 16, 36),
    "cfg4_len16": (41, 16, 132),
    "cfg4_len40": (42, 40, 132),
    "cfg4_len100": (43, 100, 132),
}
N_CFG4 = 128
SRC, TGT = "eng_Latn", "fra_Latn"


def step_margins(stderr: str):
    """Per-step reference margins from the [ref-step] lines, in step order."""
    out = []
    for m in re.finditer(r"^\[ref-step\] (\d+) (\d+)((?: \S+)*)$", stderr, re.M):
        scores = [float(x) for x in m.group(3).split()]
        lim = min(len(scores), BEAM + 1)
        gaps = [scores[i] - scores[i + 1] for i in range(lim - 1)]
        out.append((int(m.group(1)), min(gaps) if gaps else float("inf")))
    steps = [s for s, _ in out]
    assert steps == list(range(2, 2 + len(steps))), steps
    return [g for _, g in out]


def run_reference(model: str, src_ids, max_gen: int):
    exe = os.path.join(REPO, "oracle", "_ref", f"pico_nllb_g{max_gen}_steplog")
    args = [exe, model, SRC, TGT] + [str(t) for t in src_ids[1:-1]]
    t0 = time.time()
    r = subprocess.run(args, capture_output=True, text=True, check=True)
    dt = time.time() - t0
    out = r.stdout
    toks = [int(t) for t in re.search(r"^tokens:(.*)$", out, re.M).group(1).split()]
    best = re.search(r"^best: (\d+) tokens, score=([-0-9.]+), enc=(\d+)ms, dec=(\d+)ms, ([0-9.]+) tok/s", out, re.M)
    info = {"n_out": int(best.group(1)), "score_2dp": float(best.group(2)),
            "enc_ms": int(best.group(3)), "dec_ms": int(best.group(4)),
            "tok_s": float(best.group(5)), "wall_s": round(dt, 2)}
    return toks, step_margins(r.stderr), info


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("model", nargs="?", default=sm.default_model_path(0))
    ap.add_argument("--jobs", type=int, default=max(1, (os.cpu_count() or 4) // 4))
    ap.add_argument("--reuse", action="store_true", help="keep unchanged cases of the existing file")
    a = ap.parse_args()
    old = {}
    if a.reuse and os.path.exists(OUT):
        with open(OUT) as f:
            old = json.load(f)["cases"]
    sm.ensure_model(a.model, seed=0)
    subprocess.run(["make", "-C", os.path.join(REPO, "oracle"), "ref-main"], check=True)
    jobs = []
    for name, (seed, n, max_gen) in HAND_PICKED.items():
        jobs.append((name, {"seed": seed, "n_tokens": n, "max_gen": max_gen},
                     sm.source_ids(seed, n, SRC), max_gen))
    for i, src in enumerate(sm.config4_sources(N_CFG4)):
        jobs.append((f"cfg4_s{i:02d}", {"workload_index": i, "n_tokens": len(src) - 2, "max_gen": 132},
                     src, 132))

    def work(job):
        name, meta, src, max_gen = job
        prev = old.get(name)
        if prev is not None and prev["src"] == src and prev["max_gen"] == max_gen:
            return name, prev
        toks, margins, info = run_reference(a.model, src, max_gen)
        print(name, len(src), "->", len(toks), f"min margin {min(margins):.3g}", info, flush=True)
        return name, dict(meta, src=src, tokens=toks, margins=[float(f"{g:.6g}") for g in margins],
                          reference=info)

    with ThreadPoolExecutor(a.jobs) as ex:
        results = list(ex.map(work, jobs))
    res = {"model": {"generator": "nllb_attn.synth_model.write_model", "seed": 0},
           "src_lang": SRC, "tgt_lang": TGT, "tgt_lang_id": sm.LANG[TGT],
           "margin_rule": "per step from 2: min gap of consecutive sorted candidate scores among the "
                          "first BEAM_SIZE+1 (reference program, oracle/ref_steplog.h)",
           "cfg4_first": N_CFG4, "cases": dict(results)}
    cases = res.pop("cases")
    with open(OUT, "w") as f:  # one line per case
        head = json.dumps(res, indent=1)[:-2]
        body = ",\n".join(f"  {json.dumps(k)}: {json.dumps(v)}" for k, v in cases.items())
        f.write(f'{head},\n "cases": {{\n{body}\n }}\n}}\n')
    print("wrote", OUT)


if __name__ == "__main__":
    main()
