"""Regenerate tests/golden/golden_outputs.npz from the reference itself.

Runs the reference's own attention code (tensor.c / decoder.c compiled from
the reference sources into oracle/_ref/ by oracle/Makefile) and main.c's
penalty / log-softmax / top-k functions (oracle/ref_search_harness.c) on the
seeded inputs defined in cases.py and stores their outputs.  Needs the reference
sources at build time (REF_DIR, by default the reference checkout beside
this repository, oracle/Makefile); the fixtures are
committed so that nothing else ever needs them.

    python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import cases  # noqa: E402
from cases import po  # noqa: E402


def main() -> None:
    po.build(quiet=False)
    out = {}
    for name in cases.PREFILL_CASES:
        q, k, v, vl = cases.prefill_case(name)
        out[name] = po.ref_prefill_flash(q, k, v, vl)
    Q, K, V, mask = cases.head_mask_case()
    out["head_flash_mask"] = po.ref_attention_head(Q, K, V, mask, flash=True)
    out["head_mask"], out["head_mask_scores"] = po.ref_attention_head(Q, K, V, mask, flash=False,
                                                                      return_scores=True)
    for name, steps in cases.DECODE_CASES.items():
        q, k, v, parents = cases.decode_case(name)
        full = po.ref_decode_sweep(q, k, v, parents)
        out[name] = full[list(steps)]
    for name in cases.CROSS_CASES:
        K, V, q = cases.cross_case(name)
        out[name] = po.ref_cross(K, V, q)
    for name in cases.PENALTY_CASES:
        logits, tokens, lens, pen, ngram = cases.penalties_case(name)
        res = po.ref_penalties(logits, tokens, lens, pen, ngram)
        idx = np.nonzero((res != logits).reshape(-1))[0].astype(np.int64)
        out[name + "_idx"] = idx
        out[name + "_val"] = res.reshape(-1)[idx]
    for name in cases.TOPK_CASES:
        logits, k = cases.topk_case(name)
        tok, sc = po.ref_logsoftmax_topk(logits, k)
        out[name + "_tok"] = tok
        out[name + "_logp"] = sc
    for name in cases.LINEAR_CASES:
        x, w, scale, bias, rows = cases.linear_case(name)
        out[name] = po.ref_linear(x[rows], w, scale, bias)
    np.savez_compressed(cases.GOLDEN_NPZ, **out)
    for k_, v_ in out.items():
        print(f"{k_:22s} {str(v_.shape):22s} sum={float(np.sum(v_, dtype=np.float64)):+.6f}")
    print("wrote", cases.GOLDEN_NPZ, os.path.getsize(cases.GOLDEN_NPZ), "bytes")


if __name__ == "__main__":
    main()
